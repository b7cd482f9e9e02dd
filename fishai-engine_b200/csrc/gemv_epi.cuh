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

// Fused epilogue for chunk c, run by the NW*32 consumer threads of the CTA
// that completed the chunk.  Phase 1 sums the chunk's published partials into
// `sums` (shared memory, >= width floats): thread pair (2q, 2q+1) takes
// column quad q, one the first half of the contributor list and one the
// second, each in list order, 12 float4 loads in flight; the pair adds its
// two halves (a fixed order, so results are deterministic).  `sl` lists the
// contributors' partial slots (shared memory on the MMA path).  Phase 2
// applies the launch's epilogue mode to the sums.
template <int NW>
__device__ void epilogue(const GemvParams &p, float *red, float *sums, const uint32_t *sl, const ChunkDesc &cd,
                         uint32_t c, uint32_t tid, uint32_t warp, uint32_t lane) {
  constexpr uint32_t NT = NW * 32;
  constexpr uint32_t kInFlight = 12;
  const uint32_t w = cd.width, n = cd.n_contrib, nq = w / 4;
  for (uint32_t i0 = 0; i0 < 2 * nq; i0 += NT) {  // uniform trip count: pairs stay together for the shuffle
    const uint32_t i = i0 + tid, q = i >> 1, h = i & 1;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (i < 2 * nq) {
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
    if (i < 2 * nq && h == 0)
      reinterpret_cast<float4 *>(sums)[q] = make_float4(acc.x + ox, acc.y + oy, acc.z + oz, acc.w + ow);
  }
  consumer_bar<NW>();
  float local = 0.0f;
  unsigned long long best = 0ull;
  if (p.epi == kEpiSwiglu) {
    const uint32_t half = w / 2;
    for (uint32_t i = tid; i < half; i += NT) p.out[cd.out_col / 2 + i] = __fmul_rn(silu_ref(sums[i]), sums[i + half]);
  } else {
    const uint32_t pos = (p.epi == kEpiQkv) ? p.state->pos : 0;   // RoPE position
    const uint32_t wpos = (p.epi == kEpiQkv) ? p.state->len : 0;  // cache slot written
    if (p.epi == kEpiQkv && pos >= p.rope_max && tid == 0) atomicOr(&p.state->err, kErrContext);
    for (uint32_t i = tid; i < w; i += NT) {
      const float v = sums[i];
      const uint32_t col = cd.out_col + i;
      if (p.epi == kEpiStore) {
        p.out[col] = v;
      } else if (p.epi == kEpiResid) {
        const float nv = __ldcg(p.resid + col) + v;
        p.resid[col] = nv;
        local = fmaf(nv, nv, local);
      } else if (p.epi == kEpiLogits) {
        if (p.out) p.out[col] = v;
        const unsigned long long key = ((unsigned long long)float_key(v) << 32) | (unsigned long long)(~col);
        best = key > best ? key : best;
      } else {  // kEpiQkv
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
          const uint32_t page_idx = wpos / 16;
          if (page_idx < p.kv.max_pages) {
            const uint32_t page = p.kv.page_table[p.seq * p.kv.max_pages + page_idx];
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
