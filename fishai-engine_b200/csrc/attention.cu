// Decode attention over the paged KV cache (split-K "flash decode").
//
// Reference: scaled_dot_product_attention with the cache expanded per query
// head (src/model.rs:374-394, src/tensor.rs:451-551): s = (q.k)*scale,
// softmax over every cached position, o = sum p*v; GQA query head h reads kv
// head h / (H/KVH) (expand_kv_heads, src/model.rs:500-526) — no copy here,
// the kv head is indexed directly.  Grid (splits, KVH, query rows); a CTA
// handles all query heads of one kv head over one contiguous slice of
// positions, keeps an online softmax per head and writes (max, sum,
// unnormalised o) partials; the last split CTA of a kv head combines them.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "fa_dequant.cuh"
#include "fa_device.cuh"
#include "fa_kernels.hpp"

namespace fa {

namespace {
constexpr int kWarps = 4;
constexpr int kMaxRep = 8;   // query heads per kv head
constexpr int kTile = 32;    // positions per warp tile (one per lane in the score phase)
constexpr uint32_t kMaxSplits = 64;

// dynamic shared memory of one CTA: q [REP][hd] | per warp V tile [32][hd] |
// per warp p [32][REP] | merge scratch m, l [kWarps][REP], o [kWarps][REP][hd]
__host__ __device__ inline size_t attn_smem(uint32_t rep, uint32_t hd, bool f16) {
  return (size_t)rep * hd * 4 + (size_t)kWarps * kTile * hd * (f16 ? 2 : 4) + (size_t)kWarps * kTile * rep * 4 +
         (size_t)kWarps * rep * 8 + (size_t)kWarps * rep * hd * 4;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ uint4 ldg_nc(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

template <bool F16>
__device__ __forceinline__ float elem(const void *row, uint32_t d) {
  if (F16) return __half2float(reinterpret_cast<const __half *>(row)[d]);
  return reinterpret_cast<const float *>(row)[d];
}

// One CTA = (split, kv head, query row).  Warp w takes the 32-position tiles
// w, w+4, ... of the split.  Score phase: lane t owns position t of the tile
// and forms q_r . k_t for the REP query heads of the kv head from 16-byte
// loads of its K row; online softmax across tiles per warp.  The tile's V rows
// are copied to shared memory (cp.async) while the scores are computed; in
// the PV phase lane l owns dims l, l+32, ...  Warps merge in a fixed order,
// the split partial (max, sum, unnormalised o) goes to global memory and the
// last split CTA of the kv head combines all splits (fixed order).
template <bool F16, int REP>
__device__ void attn_body(const AttnParams &p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t split = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;
  const uint32_t hd = p.kv.head_dim, KVH = p.kv.n_kv, esz = F16 ? 2 : 4;
  // batched decode: row r is cache sequence row_seq0 + r with its own length
  const uint32_t T = p.kc ? p.t_fixed : (p.row_states ? p.row_states[row].len : p.state->len) + 1;
  const uint32_t seq = p.row_states ? p.row_seq0 + row : p.seq;
  const float *qrow = p.q + (uint64_t)row * p.n_heads * hd;
  float *part = p.part + (uint64_t)row * p.n_heads * p.splits * (2 + hd);
  uint32_t *counters = p.counters + (uint64_t)row * KVH;
  float *outrow = p.out + (uint64_t)row * p.n_heads * hd;
  uint32_t L = (T + p.splits - 1) / p.splits;
  L = (L + 15) / 16 * 16;
  const uint32_t t0 = min(T, split * L), t1 = min(T, t0 + L);

  float *qs = reinterpret_cast<float *>(smem_raw);                       // [REP][hd]
  uint8_t *vt = smem_raw + (size_t)REP * hd * 4;                         // [kWarps][32][hd]
  float *ps = reinterpret_cast<float *>(vt + (size_t)kWarps * kTile * hd * esz);  // [kWarps][32][REP]
  float *sm_m = ps + kWarps * kTile * REP, *sm_l = sm_m + kWarps * REP;  // [kWarps][REP]
  float *sm_o = sm_l + kWarps * REP;                                     // [kWarps][REP][hd]
  for (uint32_t i = threadIdx.x; i < REP * hd; i += blockDim.x) qs[i] = qrow[kvh * REP * hd + i];
  __syncthreads();

  const uint8_t *base = p.kc ? nullptr
                             : reinterpret_cast<const uint8_t *>(p.kv.base) + (uint64_t)p.layer * p.kv.layer_stride * esz;
  const uint32_t *pt = p.kc ? nullptr : p.kv.page_table + (uint64_t)seq * p.kv.max_pages;
  auto row_ptr = [&](uint32_t t, int is_v) -> const uint8_t * {
    if (p.kc) return reinterpret_cast<const uint8_t *>(is_v ? p.vc : p.kc) + ((uint64_t)t * KVH + kvh) * hd * 4;
    return base + kv_index(pt[t / 16], is_v, kvh, t % 16, 0, KVH, hd) * esz;
  };
  constexpr uint32_t DPL = 4;  // dims per lane in the PV phase (hd <= 128)
  float m[REP], l[REP], o[REP][DPL];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (uint32_t i = 0; i < DPL; ++i) o[r][i] = 0.0f;
  }
  uint8_t *vw = vt + (size_t)warp * kTile * hd * esz;
  float *pw = ps + warp * kTile * REP;
  const uint32_t vw_s = (uint32_t)__cvta_generic_to_shared(vw);
  const uint32_t chunks = hd * esz / 16;  // 16-byte pieces of one row
  const bool vec = (hd * esz) % 16 == 0;
  for (uint32_t tb = t0 + warp * kTile; tb < t1; tb += kWarps * kTile) {
    const uint32_t nv = min((uint32_t)kTile, t1 - tb);
    // V rows of the tile -> shared memory (asynchronous when rows are whole
    // 16-byte pieces, element by element otherwise)
    if (vec) {
      for (uint32_t i = lane; i < nv * chunks; i += 32) {
        const uint32_t tt = i / chunks, c = i % chunks;
        cp_async16(vw_s + (tt * chunks + c) * 16, row_ptr(tb + tt, 1) + c * 16);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    } else {
      for (uint32_t i = lane; i < nv * hd; i += 32) {
        const uint32_t tt = i / hd, d = i % hd;
        if (F16) reinterpret_cast<__half *>(vw)[i] = reinterpret_cast<const __half *>(row_ptr(tb + tt, 1))[d];
        else reinterpret_cast<float *>(vw)[i] = reinterpret_cast<const float *>(row_ptr(tb + tt, 1))[d];
      }
    }
    // scores: lane = position
    float s[REP];
#pragma unroll
    for (int r = 0; r < REP; ++r) s[r] = 0.0f;
    const bool valid = lane < nv;
    if (valid && !vec) {
      const uint8_t *kr = row_ptr(tb + lane, 0);
      for (uint32_t d = 0; d < hd; ++d) {
        const float kd = elem<F16>(kr, d);
#pragma unroll
        for (int r = 0; r < REP; ++r) s[r] = fmaf(qs[r * hd + d], kd, s[r]);
      }
    } else if (valid) {
      const uint8_t *kr = row_ptr(tb + lane, 0);
      for (uint32_t c0 = 0; c0 < chunks; c0 += 8) {
        uint4 kv8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (c0 + j < chunks) kv8[j] = ldg_nc(kr + (c0 + j) * 16);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (c0 + j >= chunks) break;
          const uint32_t w4[4] = {kv8[j].x, kv8[j].y, kv8[j].z, kv8[j].w};
          float kf[8];
          uint32_t nk;
          if (F16) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w4[e]));
              kf[2 * e] = f.x;
              kf[2 * e + 1] = f.y;
            }
            nk = 8;
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) kf[e] = __uint_as_float(w4[e]);
            nk = 4;
          }
          const uint32_t d0 = (c0 + j) * (F16 ? 8 : 4);
#pragma unroll
          for (int r = 0; r < REP; ++r) {
            const float4 qa = *reinterpret_cast<const float4 *>(qs + r * hd + d0);
            s[r] = fmaf(qa.x, kf[0], s[r]);
            s[r] = fmaf(qa.y, kf[1], s[r]);
            s[r] = fmaf(qa.z, kf[2], s[r]);
            s[r] = fmaf(qa.w, kf[3], s[r]);
            if (nk == 8) {
              const float4 qb = *reinterpret_cast<const float4 *>(qs + r * hd + d0 + 4);
              s[r] = fmaf(qb.x, kf[4], s[r]);
              s[r] = fmaf(qb.y, kf[5], s[r]);
              s[r] = fmaf(qb.z, kf[6], s[r]);
              s[r] = fmaf(qb.w, kf[7], s[r]);
            }
          }
        }
      }
    }
    // online softmax over the tile
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      const float sv = valid ? s[r] * p.scale : -INFINITY;
      float mt = sv;
#pragma unroll
      for (int off = 16; off; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xFFFFFFFFu, mt, off));
      const float mn = fmaxf(m[r], mt);
      const float alpha = expf(m[r] - mn);  // m[r] = -inf on the first tile: alpha = 0
      const float pv = valid ? expf(sv - mn) : 0.0f;
      float ls = pv;
#pragma unroll
      for (int off = 16; off; off >>= 1) ls += __shfl_xor_sync(0xFFFFFFFFu, ls, off);
      l[r] = fmaf(l[r], alpha, ls);
      m[r] = mn;
#pragma unroll
      for (uint32_t i = 0; i < DPL; ++i) o[r][i] *= alpha;
      pw[lane * REP + r] = pv;
    }
    if (vec) cp_async_wait_all();
    __syncwarp();
    // PV: lane owns dims lane + 32 i
    for (uint32_t tt = 0; tt < nv; ++tt) {
      float pr[REP];
#pragma unroll
      for (int r = 0; r < REP; ++r) pr[r] = pw[tt * REP + r];
      const uint8_t *vr = vw + (size_t)tt * hd * esz;
#pragma unroll
      for (uint32_t i = 0; i < DPL; ++i) {
        const uint32_t d = lane + 32 * i;
        if (d < hd) {
          const float v = elem<F16>(vr, d);
#pragma unroll
          for (int r = 0; r < REP; ++r) o[r][i] = fmaf(pr[r], v, o[r][i]);
        }
      }
    }
    __syncwarp();
  }
  // merge the warps (fixed order)
  for (uint32_t r = 0; r < REP; ++r) {
    if (lane == 0) {
      sm_m[warp * REP + r] = m[r];
      sm_l[warp * REP + r] = l[r];
    }
    for (uint32_t i = 0; i < DPL; ++i) {
      const uint32_t d = lane + 32 * i;
      if (d < hd) sm_o[(warp * REP + r) * hd + d] = o[r][i];
    }
  }
  __syncthreads();
  for (uint32_t idx = threadIdx.x; idx < REP * (hd + 2); idx += blockDim.x) {
    const uint32_t r = idx / (hd + 2), c = idx % (hd + 2);
    float M = -INFINITY;
    for (int wv = 0; wv < kWarps; ++wv) M = fmaxf(M, sm_m[wv * REP + r]);
    float out;
    if (c == 0) {
      out = M;
    } else {
      float acc = 0.0f;
      for (int wv = 0; wv < kWarps; ++wv) {
        const float mw = sm_m[wv * REP + r];
        if (mw == -INFINITY) continue;
        const float e = expf(mw - M);
        acc = fmaf(c == 1 ? sm_l[wv * REP + r] : sm_o[(wv * REP + r) * hd + c - 2], e, acc);
      }
      out = acc;
    }
    const uint32_t h = kvh * REP + r;
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
  // per query head: max over splits, weights exp(m_s - M), total sum (warp
  // reductions, fixed order); then each output dim from independent loads
  __shared__ float ecoef[kMaxRep * kMaxSplits];
  __shared__ float lsum[kMaxRep];
  for (uint32_t r = warp; r < REP; r += kWarps) {
    const float *P = part + (uint64_t)(kvh * REP + r) * p.splits * (2 + hd);
    float M = -INFINITY;
    for (uint32_t s = lane; s < p.splits; s += 32) M = fmaxf(M, __ldcg(P + s * (2 + hd)));
#pragma unroll
    for (int off = 16; off; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, off));
    float Ls = 0.0f;
    for (uint32_t s = lane; s < p.splits; s += 32) {
      const float ms = __ldcg(P + s * (2 + hd));
      const float e = ms == -INFINITY ? 0.0f : expf(ms - M);
      ecoef[r * kMaxSplits + s] = e;
      Ls = fmaf(__ldcg(P + s * (2 + hd) + 1), e, Ls);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) Ls += __shfl_xor_sync(0xFFFFFFFFu, Ls, off);
    if (lane == 0) lsum[r] = Ls;
  }
  __syncthreads();
  // output: warp per query head, lane per 4 dims; the splits' o vectors are
  // loaded 16 at a time (independent loads), summed in split order
  for (uint32_t r = warp; r < REP; r += kWarps) {
    const uint32_t h = kvh * REP + r;
    const float *P = part + (uint64_t)h * p.splits * (2 + hd) + 2;
    const float *ec = ecoef + r * kMaxSplits;
    for (uint32_t d0 = 4 * lane; d0 < hd; d0 += 128) {
      const uint32_t nd = min(4u, hd - d0);
      float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (uint32_t sp = 0; sp < p.splits; sp += 16) {
        float a[16][4];
#pragma unroll
        for (int j = 0; j < 16; ++j)
#pragma unroll
          for (uint32_t e = 0; e < 4; ++e)
            a[j][e] = (sp + j < p.splits && e < nd) ? __ldcg(P + (sp + j) * (2 + hd) + d0 + e) : 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (sp + j >= p.splits) break;
#pragma unroll
          for (uint32_t e = 0; e < 4; ++e) o[e] = fmaf(a[j][e], ec[sp + j], o[e]);
        }
      }
#pragma unroll
      for (uint32_t e = 0; e < 4; ++e)
        if (e < nd) outrow[h * hd + d0 + e] = o[e] / lsum[r];
    }
  }
  if (threadIdx.x == 0) counters[kvh] = 0;
}

template <bool F16, int REP>
__global__ void __launch_bounds__(kWarps * 32) k_attention(const AttnParams p) {
  pdl_launch_dependents();
  pdl_wait();
  attn_body<F16, REP>(p);
}

template <int REP>
void *pick(bool f16) {
  return f16 ? (void *)k_attention<true, REP> : (void *)k_attention<false, REP>;
}
void *pick_kernel(uint32_t rep, bool f16) {
  return rep == 1 ? pick<1>(f16) : rep == 2 ? pick<2>(f16) : rep == 4 ? pick<4>(f16) : rep == 8 ? pick<8>(f16) : nullptr;
}
}  // namespace

// once per device: allow the kernels' dynamic shared memory
int attention_init() {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  if (done.load() & (1ull << dev)) return 0;
  for (uint32_t rep : {1u, 2u, 4u, 8u})
    for (bool f16 : {false, true})
      if (cudaFuncSetAttribute(pick_kernel(rep, f16), cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)attn_smem(rep, 128, f16)) != cudaSuccess)
        return -1;
  if (attn_paged_init()) return -1;
  done.fetch_or(1ull << dev);
  return 0;
}

int launch_attention(const AttnParams &p, bool pdl, cudaStream_t st) {
  const uint32_t rep = p.n_heads / p.kv.n_kv, hd = p.kv.head_dim;
  const bool f16 = p.kv.f16 != 0;
  if (hd > 128 || rep > kMaxRep || p.n_heads % p.kv.n_kv || !p.splits || p.splits > kMaxSplits) return -1;
  if (attention_init()) return -1;
  if (attn_paged_supported(p)) return launch_attn_paged(p, pdl, st);  // batch-1 decode: bulk-copy tiles
  void *fn = pick_kernel(rep, f16);
  if (!fn) return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, p.kv.n_kv, p.q_rows ? p.q_rows : 1);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = attn_smem(rep, hd, f16);
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
