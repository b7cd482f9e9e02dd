// Batch-1 decode attention over the paged KV cache, staged by bulk copies.
//
// Reference: scaled_dot_product_attention for one query row
// (src/model.rs:374-394, src/tensor.rs:451-551): s = (q.k) * scale over every
// cached position, softmax, o = sum p * v; GQA query head h reads kv head
// h / (H / KVH) (expand_kv_heads, src/model.rs:500-526), indexed directly.
//
// Grid (splits, KVH): a CTA takes one contiguous, page-aligned range of
// positions for one kv head and all REP query heads of it, in tiles of 64
// positions (4 pages).  Data path: lane i of warp 0 issues two 1-D bulk
// copies for page i of a tile (its K block and its V block: 16 positions x hd,
// contiguous in the page layout) into a double-buffered shared-memory tile;
// the tile completes on one mbarrier.  Warp w owns positions 8w..8w+7 of each
// tile and lane l owns dims [l*DPL, (l+1)*DPL) (DPL = hd / 32) of q, k, v and
// o, all f32 arithmetic (f16 cache entries widen exactly).  Scores: each lane
// forms the partial dots of its dims for 8 positions x REP heads; a butterfly
// reduce-scatter across the lanes leaves every (position, head) total on one
// lane (a fixed summation tree).  Online softmax per warp and head, PV in
// registers; the warps merge in a fixed order, the split partial (max, sum,
// unnormalised o) goes to global memory; either the consumer combines the
// splits (the o projection's kProAttn prologue, partials_only) or the last
// split CTA of the kv head does, in split order.
// Raw form (qkv_raw, the decode step): q, k and v of this token arrive as the
// qkv launch's red.add sums; each CTA rotates q and the new k (RoPE, half
// split) in registers, the CTA whose range ends at position len writes the
// new k / v into its copy of the last tile before use and appends them to
// the cache at the end, so every tile can be requested before the wait for
// the qkv launch.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "fa_device.cuh"
#include "fa_kernels.hpp"

namespace fa {
namespace {

constexpr uint32_t kPW = 8;          // warps per CTA
constexpr uint32_t kPP = 8;          // positions per warp per tile
constexpr uint32_t kPT = kPW * kPP;  // positions per tile (4 pages)
constexpr uint32_t kMaxSplitsP = 64;

template <bool F16, int HD>
struct Geo {
  static constexpr uint32_t esz = F16 ? 2 : 4;
  static constexpr uint32_t DPL = HD / 32;
  static constexpr uint32_t page_bytes = 16 * HD * esz;   // one page's K (or V) block of one kv head
  static constexpr uint32_t tile_bytes = kPT * HD * esz;  // K (or V) of one tile
};

// shared memory: mbarriers + flag | scores [kPW][kPP*REP] | alpha / sums
// [kPW][REP] | 2 stages x (K, V) tiles, reused by the warp merge
// [kPW][REP][HD + 2] and the split combine coefficients
constexpr uint32_t kOffSc = 64;
template <int REP>
__host__ __device__ constexpr uint32_t off_al() { return kOffSc + kPW * kPP * REP * 4; }
template <int REP>
__host__ __device__ constexpr uint32_t off_tiles() { return (off_al<REP>() + kPW * REP * 4 + 127) / 128 * 128; }
template <bool F16, int REP, int HD>
__host__ __device__ constexpr size_t paged_smem() {
  const size_t stage = 4 * (size_t)Geo<F16, HD>::tile_bytes;
  const size_t merge = (size_t)kPW * REP * (HD + 2) * 4;
  const size_t comb = (size_t)REP * kMaxSplitsP * 4;
  size_t m = stage > merge ? stage : merge;
  m = m > comb ? m : comb;
  return off_tiles<REP>() + m;
}

__device__ __forceinline__ void load_dims(const uint8_t *row, bool f16, uint32_t lane, uint32_t dpl, float *out) {
  if (f16) {
    const __half *h = reinterpret_cast<const __half *>(row) + lane * dpl;
    if (dpl == 4) {
      const uint2 w = *reinterpret_cast<const uint2 *>(h);
      const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
      out[0] = a.x, out[1] = a.y, out[2] = b.x, out[3] = b.y;
    } else {
      const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(h));
      out[0] = a.x, out[1] = a.y;
    }
  } else {
    const float *f = reinterpret_cast<const float *>(row) + lane * dpl;
    if (dpl == 4) {
      const float4 a = *reinterpret_cast<const float4 *>(f);
      out[0] = a.x, out[1] = a.y, out[2] = a.z, out[3] = a.w;
    } else {
      const float2 a = *reinterpret_cast<const float2 *>(f);
      out[0] = a.x, out[1] = a.y;
    }
  }
}

template <bool F16, int REP, int HD>
__global__ void __launch_bounds__(kPW * 32) k_attn_paged(const AttnParams p) {
  using G = Geo<F16, HD>;
  constexpr uint32_t DPL = G::DPL, NV = kPP * REP;
  constexpr uint32_t VPL = NV >= 32 ? NV / 32 : 1;  // totals per lane after the reduce-scatter
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
  uint32_t *flag = reinterpret_cast<uint32_t *>(smem + 16);
  float *sc = reinterpret_cast<float *>(smem + kOffSc);
  float *al = reinterpret_cast<float *>(smem + off_al<REP>());
  uint8_t *tiles = smem + off_tiles<REP>();
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t split = blockIdx.x, kvh = blockIdx.y, KVH = p.kv.n_kv;

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  // early_kv (a step graph): len and the K/V rows of positions below len come
  // from earlier steps, i.e. earlier graph launches that completed before this
  // one began, so those tiles are fetched while the qkv launch is finishing;
  // the tile holding position len (written by that launch) waits for it
  if (!p.early_kv) pdl_wait();

  const uint32_t len = p.state->len;
  uint32_t T = len + 1;
  if (T > p.kv.max_pages * 16) {  // beyond the cache: the qkv launch has flagged it; read what exists
    T = p.kv.max_pages * 16;
    if (tid == 0 && split == 0 && kvh == 0) atomicOr(&p.state->err, kErrContext);
  }
  uint32_t L = (T + p.splits - 1) / p.splits;
  L = (L + 15) / 16 * 16;
  const uint32_t t0 = min(T, split * L), t1 = min(T, t0 + L);
  const uint32_t n_tiles = (t1 - t0 + kPT - 1) / kPT;
  const uint8_t *base = reinterpret_cast<const uint8_t *>(p.kv.base) + (uint64_t)p.layer * p.kv.layer_stride * G::esz;
  const uint32_t *pt = p.kv.page_table + (uint64_t)p.seq * p.kv.max_pages;

  auto issue = [&](uint32_t j) {  // warp 0: tile j into buffer j & 1
    const uint32_t pos0 = t0 + j * kPT;
    const uint32_t np = (min(t1, pos0 + kPT) - pos0 + 15) / 16;
    uint64_t *b = &bar[j & 1];
    if (lane == 0) mbar_arrive_expect_tx(b, np * 2 * G::page_bytes);
    __syncwarp();
    if (lane < np) {
      const uint32_t page = __ldg(pt + pos0 / 16 + lane);
      uint8_t *dk = tiles + (j & 1) * 2 * G::tile_bytes + lane * G::page_bytes;
      bulk_g2s(dk, base + kv_index(page, 0, kvh, 0, 0, KVH, HD) * G::esz, G::page_bytes, b);
      bulk_g2s(dk + G::tile_bytes, base + kv_index(page, 1, kvh, 0, 0, KVH, HD) * G::esz, G::page_bytes, b);
    }
  };
  const bool newest = t1 == len + 1;  // this split ends at position len
  // raw q/k/v: the row of position len is patched into its tile from
  // registers, so that tile needs nothing from the qkv launch either
  const bool raw = p.qkv_raw != nullptr;
  auto early = [&](uint32_t j) { return p.early_kv && (raw || !(newest && j + 1 == n_tiles)); };
  if (warp == 0) {
    if (n_tiles > 0 && early(0)) issue(0);
    if (n_tiles > 1 && early(1)) issue(1);
  }
  if (p.early_kv) pdl_wait();
  if (warp == 0) {
    if (n_tiles > 0 && !early(0)) issue(0);
    if (n_tiles > 1 && !early(1)) issue(1);
  }

  float q[REP][DPL], o[REP][DPL];
  float knew[DPL], vnew[DPL];  // raw mode: this token's k (rotated) and v, dims of this lane
  const float *qrow = (raw ? p.qkv_raw : p.q) + (uint64_t)kvh * REP * HD + lane * DPL;
#pragma unroll
  for (int h = 0; h < REP; ++h)
#pragma unroll
    for (uint32_t j = 0; j < DPL; ++j) {
      q[h][j] = __ldcg(qrow + h * HD + j);
      o[h][j] = 0.0f;
    }
  if (raw) {
    // RoPE, half-split (src/model.rs:367-368, src/tensor.rs rope): dim dd
    // pairs with dd +- hd/2, held by lane +- 16 at the same j; the same f32
    // steps as the qkv epilogue of the fixed-order path
    const uint32_t qd = p.n_heads * HD, pos = p.state->pos;
    const float *krow = p.qkv_raw + qd + (uint64_t)kvh * HD + lane * DPL;
#pragma unroll
    for (uint32_t j = 0; j < DPL; ++j) {
      knew[j] = __ldcg(krow + j);
      vnew[j] = __ldcg(krow + KVH * HD + j);
    }
    if (pos < p.rope_max) {
      const bool lo = lane < 16;
      const float *cs = p.rope_tab + (uint64_t)pos * HD + 2 * ((lane * DPL) % (HD / 2));
      float cth[DPL], sth[DPL];
#pragma unroll
      for (uint32_t j = 0; j < DPL; ++j) {
        cth[j] = __ldg(cs + 2 * j);
        sth[j] = __ldg(cs + 2 * j + 1);
      }
#pragma unroll
      for (uint32_t j = 0; j < DPL; ++j) {
        float pv[REP + 1];
#pragma unroll
        for (int h = 0; h < REP; ++h) pv[h] = __shfl_xor_sync(0xFFFFFFFFu, q[h][j], 16);
        pv[REP] = __shfl_xor_sync(0xFFFFFFFFu, knew[j], 16);
#pragma unroll
        for (int h = 0; h <= REP; ++h) {
          const float v = h < REP ? q[h][j] : knew[j];
          const float r = lo ? __fsub_rn(__fmul_rn(v, cth[j]), __fmul_rn(pv[h], sth[j]))
                             : __fadd_rn(__fmul_rn(pv[h], sth[j]), __fmul_rn(v, cth[j]));
          if (h < REP) q[h][j] = r;
          else knew[j] = r;
        }
      }
    } else if (tid == 0 && split == 0 && kvh == 0) {
      atomicOr(&p.state->err, kErrContext);
    }
    if (F16) {  // the cache holds f16: this step attends to the rounded values, as later steps will
#pragma unroll
      for (uint32_t j = 0; j < DPL; ++j) {
        knew[j] = __half2float(__float2half_rn(knew[j]));
        vnew[j] = __half2float(__float2half_rn(vnew[j]));
      }
    }
  }
  // raw mode: tile and row of position len in this CTA's range (newest split)
  const uint32_t j_new = newest ? (len - t0) / kPT : ~0u, r_new = newest ? (len - t0) % kPT : 0;
  float m_me = -INFINITY, l_me = 0.0f;  // lane h < REP: softmax state of head h
  bool ok = true;
  float *scw = sc + warp * NV;

  for (uint32_t j = 0; j < n_tiles; ++j) {
    const uint32_t pos_w = t0 + j * kPT + warp * kPP;  // first position of this warp in the tile
    if (ok && !mbar_wait_sleep(&bar[j & 1], (j >> 1) & 1)) ok = false;
    const uint8_t *kt = tiles + (j & 1) * 2 * G::tile_bytes + (size_t)warp * kPP * HD * G::esz;
    const uint8_t *vt = kt + G::tile_bytes;
    if (raw && ok && j == j_new && warp == r_new / kPP) {
      // the copied row of position len is stale: this token's k / v replace it
      uint8_t *kr = tiles + (j & 1) * 2 * G::tile_bytes + (size_t)r_new * HD * G::esz + lane * DPL * G::esz;
#pragma unroll
      for (uint32_t d = 0; d < DPL; ++d) {
        if (F16) {
          reinterpret_cast<__half *>(kr)[d] = __float2half_rn(knew[d]);
          reinterpret_cast<__half *>(kr + G::tile_bytes)[d] = __float2half_rn(vnew[d]);
        } else {
          reinterpret_cast<float *>(kr)[d] = knew[d];
          reinterpret_cast<float *>(kr + G::tile_bytes)[d] = vnew[d];
        }
      }
      __syncwarp();
    }
    if (ok) {
      // partial dots of this lane's dims: v[i * REP + h]
      float v[NV];
#pragma unroll
      for (uint32_t i = 0; i < kPP; ++i) {
        float k[DPL];
        load_dims(kt + (size_t)i * HD * G::esz, F16, lane, DPL, k);
#pragma unroll
        for (int h = 0; h < REP; ++h) {
          float a = 0.0f;
#pragma unroll
          for (uint32_t d = 0; d < DPL; ++d) a = fmaf(q[h][d], k[d], a);
          v[i * REP + h] = a;
        }
      }
      // butterfly reduce-scatter: after the halving stages lane l holds the
      // totals of indices l*VPL.. (NV >= 32) or l >> log2(32/NV) (NV < 32)
      uint32_t cnt = NV;
#pragma unroll
      for (uint32_t off = 16; off >= 1; off >>= 1) {
        if (cnt > 1) {
          const uint32_t half = cnt / 2;
          const bool up = (lane & off) != 0;
#pragma unroll
          for (uint32_t x = 0; x < NV / 2; ++x) {
            if (x < half) {
              const float send = up ? v[x] : v[x + half];
              const float keep = up ? v[x + half] : v[x];
              v[x] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, off);
            }
          }
          cnt = half;
        } else {
          v[0] += __shfl_xor_sync(0xFFFFFFFFu, v[0], off);
        }
      }
      if (NV >= 32) {
#pragma unroll
        for (uint32_t x = 0; x < VPL; ++x) {
          const uint32_t idx = lane * VPL + x, pos = pos_w + idx / REP;
          scw[idx] = pos < t1 ? v[x] * p.scale : -INFINITY;
        }
      } else {
        constexpr uint32_t sh = NV == 16 ? 1 : NV == 8 ? 2 : NV == 4 ? 3 : 4;
        if ((lane & ((1u << sh) - 1)) == 0) {
          const uint32_t idx = lane >> sh, pos = pos_w + idx / REP;
          scw[idx] = pos < t1 ? v[0] * p.scale : -INFINITY;
        }
      }
      __syncwarp();
      if (lane < REP) {  // online softmax of head `lane` over the warp's positions
        float mt = -INFINITY;
#pragma unroll
        for (uint32_t i = 0; i < kPP; ++i) mt = fmaxf(mt, scw[i * REP + lane]);
        const float mn = fmaxf(m_me, mt);
        const float alpha = mn == -INFINITY ? 1.0f : expf(m_me - mn);
        float ls = 0.0f;
#pragma unroll
        for (uint32_t i = 0; i < kPP; ++i) {
          const float s = scw[i * REP + lane];
          const float pv = s == -INFINITY ? 0.0f : expf(s - mn);
          scw[i * REP + lane] = pv;
          ls += pv;
        }
        l_me = fmaf(l_me, alpha, ls);
        m_me = mn;
        al[warp * REP + lane] = alpha;
      }
      __syncwarp();
#pragma unroll
      for (int h = 0; h < REP; ++h) {
        const float a = al[warp * REP + h];
#pragma unroll
        for (uint32_t d = 0; d < DPL; ++d) o[h][d] *= a;
      }
#pragma unroll
      for (uint32_t i = 0; i < kPP; ++i) {
        if (pos_w + i >= t1) break;  // rows past the cache end hold no data
        float vv[DPL];
        load_dims(vt + (size_t)i * HD * G::esz, F16, lane, DPL, vv);
#pragma unroll
        for (int h = 0; h < REP; ++h) {
          const float pr = scw[i * REP + h];
#pragma unroll
          for (uint32_t d = 0; d < DPL; ++d) o[h][d] = fmaf(pr, vv[d], o[h][d]);
        }
      }
      __syncwarp();
    }
    if (j + 2 < n_tiles) {
      __syncthreads();  // every warp is done with buffer j & 1
      if (warp == 0) issue(j + 2);
    }
  }
  if (!ok) {
    // a tile never completed: flag it, give the copies in flight a bounded
    // chance to land, and leave no partial
    if (lane == 0) atomicOr(&p.state->err, kErrWaitTimeout);
    if (tid == 0)
      for (uint32_t j = n_tiles > 2 ? n_tiles - 2 : 0; j < n_tiles; ++j) mbar_wait_sleep(&bar[j & 1], (j >> 1) & 1);
  }
  if (raw && newest && warp == 0) {
    // append this token's k / v at slot len (src/kv_cache.rs:50-54); every
    // copy of this CTA has landed, so nothing reads the row meanwhile
    if (len / 16 < p.kv.max_pages) {
      const uint32_t page = __ldg(pt + len / 16);
      const uint64_t lb = (uint64_t)p.layer * p.kv.layer_stride;
      const uint64_t ik = lb + kv_index(page, 0, kvh, len % 16, lane * DPL, KVH, HD);
      const uint64_t iv = lb + kv_index(page, 1, kvh, len % 16, lane * DPL, KVH, HD);
#pragma unroll
      for (uint32_t d = 0; d < DPL; ++d) {
        if (F16) {
          reinterpret_cast<__half *>(p.kv.base)[ik + d] = __float2half_rn(knew[d]);
          reinterpret_cast<__half *>(p.kv.base)[iv + d] = __float2half_rn(vnew[d]);
        } else {
          reinterpret_cast<float *>(p.kv.base)[ik + d] = knew[d];
          reinterpret_cast<float *>(p.kv.base)[iv + d] = vnew[d];
        }
      }
    } else if (lane == 0) {
      atomicOr(&p.state->err, kErrContext);
    }
  }
  __syncthreads();
  // merge the warps (fixed order) into the split partial
  float *mg = reinterpret_cast<float *>(tiles);  // [kPW][REP][HD + 2]
  if (lane < REP) {
    mg[(warp * REP + lane) * (HD + 2)] = m_me;
    mg[(warp * REP + lane) * (HD + 2) + 1] = l_me;
  }
#pragma unroll
  for (int h = 0; h < REP; ++h)
#pragma unroll
    for (uint32_t d = 0; d < DPL; ++d) mg[(warp * REP + h) * (HD + 2) + 2 + lane * DPL + d] = o[h][d];
  __syncthreads();
  // per head: the maximum over the warps and each warp's weight exp(m_w - M)
  // (0 for a warp that saw no position), once
  float *ew = sc;                 // [kPW][REP]
  float *Mh = sc + kPW * REP;     // [REP]
  if (tid < REP) {
    float M = -INFINITY;
#pragma unroll
    for (uint32_t w = 0; w < kPW; ++w) M = fmaxf(M, mg[(w * REP + tid) * (HD + 2)]);
#pragma unroll
    for (uint32_t w = 0; w < kPW; ++w) {
      const float mw = mg[(w * REP + tid) * (HD + 2)];
      ew[w * REP + tid] = mw == -INFINITY ? 0.0f : expf(mw - M);
    }
    Mh[tid] = M;
  }
  __syncthreads();
  float *part = p.part;
  for (uint32_t idx = tid; idx < REP * (HD + 2); idx += kPW * 32) {
    const uint32_t r = idx / (HD + 2), c = idx % (HD + 2);
    float out;
    if (c == 0) {
      out = Mh[r];
    } else {
      float acc = 0.0f;
#pragma unroll
      for (uint32_t w = 0; w < kPW; ++w) {
        const float e = ew[w * REP + r];
        if (e != 0.0f) acc = fmaf(mg[(w * REP + r) * (HD + 2) + c], e, acc);
      }
      out = acc;
    }
    part[((uint64_t)(kvh * REP + r) * p.splits + split) * (HD + 2) + c] = out;
  }
  if (p.partials_only) return;  // the o projection's prologue combines the splits
  // the last split CTA of this kv head combines all splits (fixed order)
  __threadfence();
  __syncthreads();
  if (tid == 0) *flag = atomicAdd(p.counters + kvh, 1u) + 1 == p.splits ? 1u : 0u;
  __syncthreads();
  if (!*flag) return;
  __threadfence();
  float *ecoef = reinterpret_cast<float *>(tiles);  // [REP][kMaxSplitsP]
  for (uint32_t r = warp; r < REP; r += kPW) {
    const float *P = part + (uint64_t)(kvh * REP + r) * p.splits * (HD + 2);
    float M = -INFINITY;
    for (uint32_t s = lane; s < p.splits; s += 32) M = fmaxf(M, __ldcg(P + s * (HD + 2)));
#pragma unroll
    for (int off = 16; off; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, off));
    float Ls = 0.0f;
    for (uint32_t s = lane; s < p.splits; s += 32) {
      const float ms = __ldcg(P + s * (HD + 2));
      const float e = ms == -INFINITY ? 0.0f : expf(ms - M);
      ecoef[r * kMaxSplitsP + s] = e;
      Ls = fmaf(__ldcg(P + s * (HD + 2) + 1), e, Ls);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) Ls += __shfl_xor_sync(0xFFFFFFFFu, Ls, off);
    if (lane == 0) al[r] = Ls;
  }
  __syncthreads();
  for (uint32_t idx = tid; idx < REP * HD; idx += kPW * 32) {
    const uint32_t r = idx / HD, d = idx % HD;
    const float *P = part + (uint64_t)(kvh * REP + r) * p.splits * (HD + 2) + 2 + d;
    const float *ec = ecoef + r * kMaxSplitsP;
    float acc = 0.0f;
    for (uint32_t s0 = 0; s0 < p.splits; s0 += 16) {
      float a[16];
#pragma unroll
      for (uint32_t x = 0; x < 16; ++x) a[x] = s0 + x < p.splits ? __ldcg(P + (s0 + x) * (HD + 2)) : 0.0f;
#pragma unroll
      for (uint32_t x = 0; x < 16; ++x)
        if (s0 + x < p.splits) acc = fmaf(a[x], ec[s0 + x], acc);
    }
    p.out[(kvh * REP + r) * HD + d] = acc / al[r];
  }
  if (tid == 0) p.counters[kvh] = 0;
}

template <bool F16, int REP, int HD>
int launch_one(const AttnParams &p, bool pdl, cudaStream_t st) {
  constexpr size_t smem = paged_smem<F16, REP, HD>();
  static_assert(smem <= 227 * 1024, "paged attention tile does not fit");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, p.kv.n_kv, 1);
  cfg.blockDim = dim3(kPW * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_attn_paged<F16, REP, HD>, p) == cudaSuccess ? 0 : -1;
}

template <bool F16, int REP, int HD>
int init_one() {
  return cudaFuncSetAttribute(k_attn_paged<F16, REP, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)paged_smem<F16, REP, HD>()) == cudaSuccess
             ? 0
             : -1;
}

template <bool F16, int HD>
int dispatch_rep(const AttnParams &p, uint32_t rep, bool pdl, cudaStream_t st) {
  switch (rep) {
    case 1: return launch_one<F16, 1, HD>(p, pdl, st);
    case 2: return launch_one<F16, 2, HD>(p, pdl, st);
    case 4: return launch_one<F16, 4, HD>(p, pdl, st);
    case 8: return launch_one<F16, 8, HD>(p, pdl, st);
    default: return -1;
  }
}

template <bool F16, int HD>
int init_rep() {
  return init_one<F16, 1, HD>() || init_one<F16, 2, HD>() || init_one<F16, 4, HD>() || init_one<F16, 8, HD>();
}

}  // namespace

bool attn_paged_supported(const AttnParams &p) {
  const uint32_t hd = p.kv.head_dim, kvh = p.kv.n_kv;
  const uint32_t rep = kvh ? p.n_heads / kvh : 0;
  return !p.kc && p.q_rows == 1 && !p.row_states && p.state && (hd == 64 || hd == 128) && kvh &&
         p.n_heads % kvh == 0 && (rep == 1 || rep == 2 || rep == 4 || rep == 8) && p.splits >= 1 &&
         p.splits <= kMaxSplitsP;
}

int attn_paged_init() {
  return init_rep<true, 64>() || init_rep<true, 128>() || init_rep<false, 64>() || init_rep<false, 128>();
}

int launch_attn_paged(const AttnParams &p, bool pdl, cudaStream_t st) {
  if (!attn_paged_supported(p)) return -1;
  const uint32_t rep = p.n_heads / p.kv.n_kv;
  if (p.kv.f16) return p.kv.head_dim == 64 ? dispatch_rep<true, 64>(p, rep, pdl, st) : dispatch_rep<true, 128>(p, rep, pdl, st);
  return p.kv.head_dim == 64 ? dispatch_rep<false, 64>(p, rep, pdl, st) : dispatch_rep<false, 128>(p, rep, pdl, st);
}

}  // namespace fa
