// Persistent decode step: one launch runs every phase of one token — the
// embedding gather, then per layer the fused QKV GEMV (RMSNorm, RoPE, KV
// append), attention, the o-projection (+ residual), the fused gate/up GEMV
// (RMSNorm, SwiGLU) and the down projection (+ residual), then the output head
// (RMSNorm, logits, argmax) — ModelWeights::forward for one token
// (src/model.rs:316-455) followed by the greedy pick (src/sampling.rs:297-310).
//
// One CTA per SM (cooperative launch: all CTAs are resident).  The producer
// lane of each CTA streams the weight stages of every GEMV phase of the step
// through one shared-memory ring without ever waiting on activations (weights
// are static), so HBM stays busy across phase boundaries.  The consumer warps
// walk the same phase list; a phase first waits until the phase it reads from
// has completed everywhere (a global counter per phase: +1 per finished GEMV
// chunk, attention kv head or embedding slice; counters grow monotonically and
// a phase of step e waits for (e + 1) x its count, so nothing is reset).  The
// last CTA to finish does the step bookkeeping (token <- argmax, positions).
// Every wait is bounded by wall time; on expiry the CTA skips the remaining
// work and raises the timeout flag for the host.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <string>

#include "fa_dequant.cuh"
#include "gemv_mma.cuh"

namespace fa {

using namespace mma;

namespace {

constexpr uint32_t kAbort = 100;  // sm.red word: a wait of this CTA expired

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ldcg128(const void *p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldcg64(const void *p) {
  uint2 v;
  asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ void group_bar(uint32_t id) { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }

// Wait (consumer thread 0, then the consumers) until done[dep] >= target.
__device__ __forceinline__ bool wait_phase(const StepParams &sp, const StepPhase &ph, uint32_t epoch, const Smem &sm,
                                           uint32_t tid) {
  if (ph.dep != ~0u && tid == 0 && !reinterpret_cast<volatile uint32_t *>(sm.red)[kAbort]) {
    const uint32_t target = (epoch + 1) * ph.dep_count;
    const uint64_t t0 = global_ns();
    while (ld_acquire(sp.done + ph.dep) < target) {
      __nanosleep(64);
      if (global_ns() - t0 > kWaitLimitNs) {
        reinterpret_cast<volatile uint32_t *>(sm.red)[kAbort] = 1u;
        break;
      }
    }
    __threadfence();
  }
  epi::consumer_bar<kWarps>();
  return !reinterpret_cast<volatile uint32_t *>(sm.red)[kAbort];
}

// embedding row slice of this CTA (src/model.rs:338-343) + its sum of squares
__device__ __forceinline__ void embed_phase(const StepParams &sp, const Smem &sm, uint32_t tid, uint32_t warp, uint32_t lane,
                            uint32_t *done) {
  const EmbedParams &p = sp.embed;
  const uint32_t fed = p.state->fed;
  uint32_t tok = (p.feed && fed < p.state->n_feed) ? p.feed[fed] : p.state->token;
  if (tok >= p.vocab) {
    if (tid == 0 && blockIdx.x == 0) atomicOr(&p.state->err, kErrBadToken);
    tok = 0;
  }
  if (tid == 0 && blockIdx.x == 0) p.state->argmax_key = 0ull;
  const uint32_t per = (p.d + gridDim.x - 1) / gridDim.x;
  const uint32_t c0 = min(p.d, blockIdx.x * per), c1 = min(p.d, c0 + per);
  float s = 0.0f;
  for (uint32_t i = c0 + tid; i < c1; i += kWarps * 32) {
    const float v = dequant_native_elem(p.type, p.emb, (uint64_t)tok * p.d + i);
    p.x[i] = v;
    s = fmaf(v, v, s);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  if (lane == 0) sm.red[warp] = s;
  epi::consumer_bar<kWarps>();
  if (tid == 0) {
    float t = 0.0f;
    for (int i = 0; i < kWarps; ++i) t += sm.red[i];
    p.ssq_out[blockIdx.x] = t;
    __threadfence();
    atomicAdd(done, 1u);
  }
  epi::consumer_bar<kWarps>();
}

// scratch of one attention work group (floats): q [REP][hd] | p [4][32][REP] |
// m, l [4][REP] | o [4][REP][hd] | e [REP][64] | lsum [REP] | flag
__host__ __device__ inline uint32_t attn_scratch_floats(uint32_t rep, uint32_t hd) {
  return rep * hd + 4 * 32 * rep + 8 * rep + 4 * rep * hd + 64 * rep + rep + 4;
}

// One (split, kv head) item of decode attention by a group of 4 warps
// (src/tensor.rs:451-551 with the GQA head mapping of src/model.rs:500-526):
// lane-per-position scores from 16-byte K loads, per-warp online softmax,
// PV with each lane owning 4 dims, merge of the 4 warps, the split partial,
// and — for the last split of the kv head — the combine into attn_out.
template <bool F16, int REP>
__device__ __forceinline__ void attn_item(const AttnParams &p, uint32_t split, uint32_t kvh, uint32_t gwarp, uint32_t lane,
                          uint32_t bar, float *scr, uint32_t *done) {
  const uint32_t gtid = gwarp * 32 + lane;
  const uint32_t hd = p.kv.head_dim, KVH = p.kv.n_kv, esz = F16 ? 2 : 4;
  const uint32_t T = p.state->len + 1;
  uint32_t L = (T + p.splits - 1) / p.splits;
  L = (L + 15) / 16 * 16;
  const uint32_t t0 = min(T, split * L), t1 = min(T, t0 + L);
  float *qs = scr, *pw = qs + REP * hd + gwarp * 32 * REP;
  float *mm = qs + REP * hd + 4 * 32 * REP, *ll = mm + 4 * REP, *oo = ll + 4 * REP;
  float *ecoef = oo + 4 * REP * hd, *lsum = ecoef + 64 * REP;
  uint32_t *flag = reinterpret_cast<uint32_t *>(lsum + REP);
  for (uint32_t i = gtid; i < REP * hd; i += 128) qs[i] = __ldcg(p.q + kvh * REP * hd + i);
  group_bar(bar);
  const uint8_t *base = reinterpret_cast<const uint8_t *>(p.kv.base) + (uint64_t)p.layer * p.kv.layer_stride * esz;
  const uint32_t *pt = p.kv.page_table + (uint64_t)p.seq * p.kv.max_pages;
  auto row_ptr = [&](uint32_t t, int is_v) -> const uint8_t * {
    return base + kv_index(pt[t / 16], is_v, kvh, t % 16, 0, KVH, hd) * esz;
  };
  const uint32_t chunks = hd * esz / 16, d0 = 4 * lane;
  float m[REP], l[REP], o[REP][4];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) o[r][i] = 0.0f;
  }
  for (uint32_t tb = t0 + gwarp * 32; tb < t1; tb += 128) {
    const uint32_t nv = min(32u, t1 - tb);
    const bool valid = lane < nv;
    float s[REP];
#pragma unroll
    for (int r = 0; r < REP; ++r) s[r] = 0.0f;
    if (valid) {
      const uint8_t *kr = row_ptr(tb + lane, 0);
      for (uint32_t c0 = 0; c0 < chunks; c0 += 4) {
        uint4 kv8[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (c0 + j < chunks) kv8[j] = ldcg128(kr + (c0 + j) * 16);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (c0 + j >= chunks) break;
          const uint32_t w4[4] = {kv8[j].x, kv8[j].y, kv8[j].z, kv8[j].w};
          float kf[8];
          if (F16) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w4[e]));
              kf[2 * e] = f.x;
              kf[2 * e + 1] = f.y;
            }
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) kf[e] = __uint_as_float(w4[e]);
          }
          const uint32_t dq = (c0 + j) * (F16 ? 8 : 4);
#pragma unroll
          for (int r = 0; r < REP; ++r) {
            const float4 qa = *reinterpret_cast<const float4 *>(qs + r * hd + dq);
            s[r] = fmaf(qa.x, kf[0], s[r]);
            s[r] = fmaf(qa.y, kf[1], s[r]);
            s[r] = fmaf(qa.z, kf[2], s[r]);
            s[r] = fmaf(qa.w, kf[3], s[r]);
            if (F16) {
              const float4 qb = *reinterpret_cast<const float4 *>(qs + r * hd + dq + 4);
              s[r] = fmaf(qb.x, kf[4], s[r]);
              s[r] = fmaf(qb.y, kf[5], s[r]);
              s[r] = fmaf(qb.z, kf[6], s[r]);
              s[r] = fmaf(qb.w, kf[7], s[r]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < REP; ++r) {
      const float sv = valid ? s[r] * p.scale : -INFINITY;
      float mt = sv;
#pragma unroll
      for (int off = 16; off; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xFFFFFFFFu, mt, off));
      const float mn = fmaxf(m[r], mt);
      const float alpha = expf(m[r] - mn);
      const float pv = valid ? expf(sv - mn) : 0.0f;
      float ls = pv;
#pragma unroll
      for (int off = 16; off; off >>= 1) ls += __shfl_xor_sync(0xFFFFFFFFu, ls, off);
      l[r] = fmaf(l[r], alpha, ls);
      m[r] = mn;
#pragma unroll
      for (int i = 0; i < 4; ++i) o[r][i] *= alpha;
      pw[lane * REP + r] = pv;
    }
    __syncwarp();
    // PV: lane owns dims d0..d0+3; V rows loaded four at a time
    if (d0 < hd) {
      for (uint32_t t8 = 0; t8 < nv; t8 += 4) {
        float vv[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (t8 + j < nv) {
            const uint8_t *vr = row_ptr(tb + t8 + j, 1) + d0 * esz;
            if (F16) {
              const uint2 h = ldcg64(vr);
              const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&h.x));
              const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&h.y));
              vv[j][0] = a.x;
              vv[j][1] = a.y;
              vv[j][2] = b.x;
              vv[j][3] = b.y;
            } else {
              const uint4 f = ldcg128(vr);
              vv[j][0] = __uint_as_float(f.x);
              vv[j][1] = __uint_as_float(f.y);
              vv[j][2] = __uint_as_float(f.z);
              vv[j][3] = __uint_as_float(f.w);
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (t8 + j >= nv) break;
#pragma unroll
          for (int r = 0; r < REP; ++r) {
            const float pr = pw[(t8 + j) * REP + r];
#pragma unroll
            for (int i = 0; i < 4; ++i) o[r][i] = fmaf(pr, vv[j][i], o[r][i]);
          }
        }
      }
    }
    __syncwarp();
  }
  // merge the group's warps (fixed order) into the split partial
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    if (lane == 0) {
      mm[gwarp * REP + r] = m[r];
      ll[gwarp * REP + r] = l[r];
    }
    if (d0 < hd)
#pragma unroll
      for (int i = 0; i < 4; ++i) oo[(gwarp * REP + r) * hd + d0 + i] = o[r][i];
  }
  group_bar(bar);
  float *part = p.part;
  for (uint32_t idx = gtid; idx < REP * (hd + 2); idx += 128) {
    const uint32_t r = idx / (hd + 2), c = idx % (hd + 2);
    float M = -INFINITY;
    for (int wv = 0; wv < 4; ++wv) M = fmaxf(M, mm[wv * REP + r]);
    float out;
    if (c == 0) {
      out = M;
    } else {
      float acc = 0.0f;
      for (int wv = 0; wv < 4; ++wv) {
        const float mw = mm[wv * REP + r];
        if (mw == -INFINITY) continue;
        const float e = expf(mw - M);
        acc = fmaf(c == 1 ? ll[wv * REP + r] : oo[(wv * REP + r) * hd + c - 2], e, acc);
      }
      out = acc;
    }
    part[((uint64_t)(kvh * REP + r) * p.splits + split) * (2 + hd) + c] = out;
  }
  __threadfence();
  group_bar(bar);
  if (gtid == 0) *flag = atomicAdd(p.counters + kvh, 1u) + 1 == p.splits ? 1u : 0u;
  group_bar(bar);
  if (!*flag) return;
  __threadfence();
  // the last split of this kv head: combine all splits (fixed order)
  for (uint32_t r = gwarp; r < REP; r += 4) {
    const float *P = part + (uint64_t)(kvh * REP + r) * p.splits * (2 + hd);
    float M = -INFINITY;
    for (uint32_t sp = lane; sp < p.splits; sp += 32) M = fmaxf(M, __ldcg(P + sp * (2 + hd)));
#pragma unroll
    for (int off = 16; off; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, off));
    float Ls = 0.0f;
    for (uint32_t sp = lane; sp < p.splits; sp += 32) {
      const float ms = __ldcg(P + sp * (2 + hd));
      const float e = ms == -INFINITY ? 0.0f : expf(ms - M);
      ecoef[r * 64 + sp] = e;
      Ls = fmaf(__ldcg(P + sp * (2 + hd) + 1), e, Ls);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) Ls += __shfl_xor_sync(0xFFFFFFFFu, Ls, off);
    if (lane == 0) lsum[r] = Ls;
  }
  group_bar(bar);
  for (uint32_t r = gwarp; r < REP; r += 4) {
    const uint32_t h = kvh * REP + r;
    const float *P = part + (uint64_t)h * p.splits * (2 + hd) + 2;
    for (uint32_t dd = d0; dd < hd; dd += 128) {
      const uint32_t nd = min(4u, hd - dd);
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (uint32_t sp = 0; sp < p.splits; sp += 4) {
        float a[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (uint32_t e = 0; e < 4; ++e)
            a[j][e] = (sp + j < p.splits && e < nd) ? __ldcg(P + (sp + j) * (2 + hd) + dd + e) : 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (sp + j >= p.splits) break;
#pragma unroll
          for (uint32_t e = 0; e < 4; ++e) acc[e] = fmaf(a[j][e], ecoef[r * 64 + sp + j], acc[e]);
        }
      }
#pragma unroll
      for (uint32_t e = 0; e < 4; ++e)
        if (e < nd) p.out[h * hd + dd + e] = acc[e] / lsum[r];
    }
  }
  if (gtid == 0) p.counters[kvh] = 0;
  __threadfence();
  group_bar(bar);
  if (gtid == 0) atomicAdd(done, 1u);
}

}  // namespace

template <bool F16, int REP>
__global__ void __launch_bounds__(kThreads, 1) k_step(const StepParams sp) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Smem sm = carve(smem, sp.gemv[0]);  // every GEMV phase shares the ring geometry
  const uint32_t tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  if (tid == 0) {
    for (uint32_t i = 0; i < sp.n_stages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kWarps);
    }
    fence_mbar_init();
    sm.red[kAbort] = 0.0f;
    reinterpret_cast<uint32_t *>(sm.red)[kAbort + 1] = ld_acquire(sp.sync);  // steps completed
  }
  for (uint32_t i = tid; i < kZeroWords; i += kThreads) sm.zero[i] = 0u;
  __syncthreads();
  const uint32_t epoch = reinterpret_cast<uint32_t *>(sm.red)[kAbort + 1];
  bool ok = true;
  if (warp == kWarps) {
    // producer: the weight stages of every GEMV phase, in phase order
    uint32_t s = 0;
    if (lane == 0)
      for (uint32_t q = 0; q < sp.n_phases && ok; ++q)
        if (sp.phases[q].kind == kPhGemv) produce(sp.gemv[sp.phases[q].idx], blockIdx.x, sm, s, ok);
    __syncwarp();  // reconverge the producer warp before the final block barrier
  } else {
    uint32_t slot = 0, phase = 0;
    constexpr uint32_t rep = REP;
    for (uint32_t q = 0; q < sp.n_phases; ++q) {
      const StepPhase ph = sp.phases[q];
      if (ph.kind == kPhEmbed) {
        if (wait_phase(sp, ph, epoch, sm, tid)) embed_phase(sp, sm, tid, warp, lane, sp.done + q);
      } else if (ph.kind == kPhGemv) {
        const GemvParams &p = sp.gemv[ph.idx];
        if (!cta_units(p, blockIdx.x)) continue;
        if (!wait_phase(sp, ph, epoch, sm, tid)) ok = false;
        consume<false>(p, blockIdx.x, sm, tid, warp, lane, slot, phase, ok);
      } else {  // attention of layer ph.idx: items (split, kv head) over (CTA, group)
        const uint32_t n_items = sp.attn.splits * sp.attn.kv.n_kv, slots = gridDim.x * sp.attn_groups;
        if (blockIdx.x * sp.attn_groups >= n_items) continue;
        if (!wait_phase(sp, ph, epoch, sm, tid)) continue;
        const uint32_t grp = warp / 4;
        if (grp < sp.attn_groups) {
          AttnParams ap = sp.attn;
          ap.layer = ph.idx;
          float *scr = reinterpret_cast<float *>(sm.tbl) + grp * attn_scratch_floats(rep, ap.kv.head_dim);
          for (uint32_t it = blockIdx.x * sp.attn_groups + grp; it < n_items; it += slots) {
            const uint32_t kvh = it / ap.splits, split = it % ap.splits;
            attn_item<F16, REP>(ap, split, kvh, warp % 4, lane, 2 + grp, scr, sp.done + q);
          }
        }
        epi::consumer_bar<kWarps>();  // the scratch overlays the GEMV tables and x slice
      }
    }
  }
  if (!ok || reinterpret_cast<volatile uint32_t *>(sm.red)[kAbort]) atomicOr(&sp.attn.state->err, kErrWaitTimeout);
  // the last CTA to finish does the step bookkeeping (k_step_end's rules)
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const uint32_t old = atomicAdd(sp.sync + 1, 1u);
    if (old + 1 == (epoch + 1) * gridDim.x) {
      __threadfence();
      SeqState *st = sp.attn.state;
      const unsigned long long key = *reinterpret_cast<volatile unsigned long long *>(&st->argmax_key);
      const uint32_t tok = ~(uint32_t)(key & 0xFFFFFFFFull);
      st->token = tok;
      if (sp.ids && st->step < sp.max_ids) sp.ids[st->step] = tok;
      st->step += 1;
      st->pos += 1;
      st->len += 1;
      if (st->fed < st->n_feed) st->fed += 1;
      __threadfence();
      atomicExch(sp.sync, epoch + 1);
    }
  }
}

namespace {
template <int REP>
void *pick_step(bool f16) { return f16 ? (void *)k_step<true, REP> : (void *)k_step<false, REP>; }
void *step_kernel(uint32_t rep, bool f16) {
  return rep == 1 ? pick_step<1>(f16) : rep == 2 ? pick_step<2>(f16) : rep == 4 ? pick_step<4>(f16)
                                       : rep == 8 ? pick_step<8>(f16) : nullptr;
}
}  // namespace

std::string step_occupancy_report(const StepParams &p, size_t smem) {
  void *fn = step_kernel(p.attn.n_heads / p.attn.kv.n_kv, p.attn.kv.f16 != 0);
  int n = -1;
  cudaFuncAttributes fa{};
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kThreads, smem);
  cudaFuncGetAttributes(&fa, fn);
  return "blocks/SM " + std::to_string(n) + ", regs " + std::to_string(fa.numRegs) + ", static smem " +
         std::to_string(fa.sharedSizeBytes) + ", max dynamic smem " + std::to_string(fa.maxDynamicSharedSizeBytes);
}

int step_attn_group_bytes(uint32_t rep, uint32_t hd) { return (int)(attn_scratch_floats(rep, hd) * 4); }


int step_init() {
  for (uint32_t rep : {1u, 2u, 4u, 8u})
    for (bool f16 : {false, true})
      if (cudaFuncSetAttribute(step_kernel(rep, f16), cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
          cudaSuccess)
        return -1;
  return 0;
}

int launch_step(const StepParams &p, size_t smem, cudaStream_t st) {
  void *fn = step_kernel(p.attn.n_heads / p.attn.kv.n_kv, p.attn.kv.f16 != 0);
  if (!fn) return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_ctas);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the phase waits need it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void *args[] = {(void *)&p};
  return (int)cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace fa
