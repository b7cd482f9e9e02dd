// Fused GEMV epilogues shared by the GEMV kernels: the last CTA to finish a
// chunk sums the chunk's published partials in a fixed contributor order
// (deterministic) and applies the epilogue mode of the launch.
#pragma once
#include <cuda_fp16.h>

#include "fa_device.cuh"
#include "fa_kernels.hpp"

namespace fa {
namespace epi {

// named barrier 1 over the NW consumer warps (the producer warp never joins)
template <int NW>
__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, %0;" ::"n"(NW * 32) : "memory"); }

__device__ __forceinline__ float silu_ref(float g) { return g * (1.0f / (1.0f + expf(-g))); }

// RoPE position and cache slot of a qkv launch, read by the consumers'
// prologue into `red` (kQkvPos, kQkvSlot) so the epilogue has them at hand.
constexpr uint32_t kQkvPos = 104, kQkvSlot = 105;

// Fused epilogue for chunk c, run by the NW*32 consumer threads of the CTA
// that completed the chunk.  Thread pair (2q, 2q+1) sums column quad q of
// the chunk's published partials, one the first half of the contributor
// list and one the second, each in list order, 12 float4 loads in flight;
// the pair adds its two halves (a fixed order, so results are deterministic).
// `sl` lists the contributors' partial slots (shared memory on the MMA path).
// Store, residual and logits launches finish in the pair's first thread with
// the quad in registers (the residual quad is fetched together with the
// partials); SwiGLU and qkv pair up columns of other quads and go through
// `sums` (shared memory, >= width floats).  qkv_smem: the kQkv* values are
// in `red` (qkv_state_prefetch), else they are read here.
template <int NW>
__device__ void epilogue(const GemvParams &p, float *red, float *sums, const uint32_t *sl, const ChunkDesc &cd,
                         uint32_t c, uint32_t tid, uint32_t warp, uint32_t lane, bool qkv_smem = false) {
  constexpr uint32_t NT = NW * 32;
  constexpr uint32_t kInFlight = 12;
  const uint32_t w = cd.width, n = cd.n_contrib, nq = w / 4;
  const bool direct = p.epi == kEpiStore || p.epi == kEpiResid || p.epi == kEpiLogits;
  // qkv: the cache page of this step's slot, fetched together with the partials
  uint32_t pos = 0, wpos = 0, page = ~0u;
  if (p.epi == kEpiQkv) {
    const uint32_t *rq = reinterpret_cast<const uint32_t *>(red);
    pos = qkv_smem ? rq[kQkvPos] : p.state->pos;     // RoPE position
    wpos = qkv_smem ? rq[kQkvSlot] : p.state->len;   // cache slot written
    if (wpos / 16 < p.kv.max_pages) page = p.kv.page_table[p.seq * p.kv.max_pages + wpos / 16];
  }
  float local = 0.0f;
  unsigned long long best = 0ull;
  for (uint32_t i0 = 0; i0 < 2 * nq; i0 += NT) {  // uniform trip count: pairs stay together for the shuffle
    const uint32_t i = i0 + tid, q = i >> 1, h = i & 1;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f), r4 = acc;
    if (i < 2 * nq) {
      if (p.epi == kEpiResid && h == 0) r4 = __ldcg(reinterpret_cast<const float4 *>(p.resid + cd.out_col) + q);
      const uint32_t lo = h ? n / 2 : 0, hi = h ? n : n / 2;
      const float4 *base = reinterpret_cast<const float4 *>(p.part) + q;
      for (uint32_t t = lo; t < hi; t += kInFlight) {
        float4 a[kInFlight];
#pragma unroll
        for (uint32_t j = 0; j < kInFlight; ++j)
          a[j] = t + j < hi ? __ldcg(base + (size_t)sl[t + j] * (p.CW / 4)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (uint32_t j = 0; j < kInFlight; ++j) {
          acc.x += a[j].x;
          acc.y += a[j].y;
          acc.z += a[j].z;
          acc.w += a[j].w;
        }
      }
    }
    const float ox = __shfl_xor_sync(0xFFFFFFFFu, acc.x, 1), oy = __shfl_xor_sync(0xFFFFFFFFu, acc.y, 1);
    const float oz = __shfl_xor_sync(0xFFFFFFFFu, acc.z, 1), ow = __shfl_xor_sync(0xFFFFFFFFu, acc.w, 1);
    if (i < 2 * nq && h == 0) {
      const float4 v = make_float4(acc.x + ox, acc.y + oy, acc.z + oz, acc.w + ow);
      const uint32_t col = cd.out_col + 4 * q;
      if (!direct) {
        reinterpret_cast<float4 *>(sums)[q] = v;
      } else if (p.epi == kEpiStore) {
        *reinterpret_cast<float4 *>(p.out + col) = v;
      } else if (p.epi == kEpiResid) {
        const float4 nv = make_float4(r4.x + v.x, r4.y + v.y, r4.z + v.z, r4.w + v.w);
        *reinterpret_cast<float4 *>(p.resid + col) = nv;
        local = fmaf(nv.x, nv.x, local);
        local = fmaf(nv.y, nv.y, local);
        local = fmaf(nv.z, nv.z, local);
        local = fmaf(nv.w, nv.w, local);
      } else {  // kEpiLogits
        if (p.out) *reinterpret_cast<float4 *>(p.out + col) = v;
        const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (uint32_t k = 0; k < 4; ++k) {
          const unsigned long long key = ((unsigned long long)float_key(e[k]) << 32) | (unsigned long long)(~(col + k));
          best = key > best ? key : best;
        }
      }
    }
  }
  if (!direct) {
    consumer_bar<NW>();
    if (p.epi == kEpiSwiglu) {
      const uint32_t half = w / 2;
      for (uint32_t i = tid; i < half; i += NT) p.out[cd.out_col / 2 + i] = __fmul_rn(silu_ref(sums[i]), sums[i + half]);
    } else {  // kEpiQkv
      const uint32_t page_idx = wpos / 16;
      if (pos >= p.rope_max && tid == 0) atomicOr(&p.state->err, kErrContext);
      for (uint32_t i = tid; i < w; i += NT) {
        const float v = sums[i];
        const uint32_t col = cd.out_col + i;
        const uint32_t hd = p.kv.head_dim, half = hd / 2;
        const bool is_q = col < p.q_dim, is_k = !is_q && col < p.q_dim + p.kv_dim;
        float outv = v;
        if ((is_q || is_k) && pos < p.rope_max) {
          const uint32_t dd = (is_q ? col : col - p.q_dim) % hd;
          const float pv = sums[dd < half ? i + half : i - half];  // partner column (same chunk)
          const float *cs = p.rope_tab + (uint64_t)pos * hd + 2 * (dd % half);
          const float cth = cs[0], sth = cs[1];
          outv = dd < half ? __fsub_rn(__fmul_rn(v, cth), __fmul_rn(pv, sth))
                           : __fadd_rn(__fmul_rn(pv, sth), __fmul_rn(v, cth));
        }
        if (is_q) {
          p.out[col] = outv;
        } else {
          const uint32_t kc = is_k ? col - p.q_dim : col - p.q_dim - p.kv_dim;
          if (page_idx < p.kv.max_pages) {
            const uint64_t idx = (uint64_t)p.layer * p.kv.layer_stride +
                                 kv_index(page, is_k ? 0 : 1, kc / hd, wpos % 16, kc % hd, p.kv.n_kv, hd);
            if (p.kv.f16) reinterpret_cast<__half *>(p.kv.base)[idx] = __float2half_rn(outv);
            else reinterpret_cast<float *>(p.kv.base)[idx] = outv;
          } else if (p.state) {
            atomicOr(&p.state->err, kErrContext);
          }
        }
      }
    }
  }
  if (p.epi == kEpiResid || p.epi == kEpiLogits) {
    for (int o = 16; o; o >>= 1) {
      local += __shfl_xor_sync(0xFFFFFFFFu, local, o);
      const unsigned long long ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
      best = ob > best ? ob : best;
    }
    unsigned long long *rk = reinterpret_cast<unsigned long long *>(red + 32);
    if (lane == 0) {
      red[warp] = local;
      rk[warp] = best;
    }
    consumer_bar<NW>();
    if (tid == 0) {
      float s = 0.0f;
      unsigned long long b = 0ull;
      for (int i = 0; i < NW; ++i) {
        s += red[i];
        b = rk[i] > b ? rk[i] : b;
      }
      if (p.epi == kEpiResid) p.ssq_out[c] = s;
      else if (p.state && b) atomicMax(&p.state->argmax_key, b);
    }
  }
  consumer_bar<NW>();  // sums is reused by the caller
}

}  // namespace epi
}  // namespace fa
