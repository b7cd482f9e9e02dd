// Token-parallel forward pieces for prefill and batched steps (the f16
// tensor-core path; ModelWeights::forward, src/model.rs:316-455, per token):
//   k_embed_rows      X[t] = E[tok[t]] (src/model.rs:338-343)
//   k_norm_rows_h     Xn[t] = f16(rms_norm(X[t]) * w) (src/tensor.rs:280-290)
//   k_rope_kv_rows    RoPE of q and k (half split, src/model.rs:469-491), K/V
//                     appended to the paged cache, q to f16 for attention
//   k_attn_causal     causal flash attention over the paged cache: token t
//                     sees cache slots [0, len0 + t] (the sequential forwards
//                     of a prompt), GQA by index; mma.sync f16, f32 softmax
//   k_swiglu_rows     H[t] = f16(silu(gate) * up) from the interleaved
//                     gate/up GEMM output (src/model.rs:413-420)
//   k_last_row        the last token's hidden state and its sum of squares
//                     into the decode workspace for the output head
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "fa_dequant.cuh"
#include "fa_device.cuh"
#include "fa_kernels.hpp"

namespace fa {
namespace {

__global__ void k_embed_rows(const uint8_t *emb, int type, const uint32_t *tok, uint32_t T, uint32_t d, uint32_t vocab,
                             float *x, uint32_t *err) {
  pdl_enter();
  const uint32_t t = blockIdx.x;
  if (t >= T) return;
  uint32_t id = tok[t];
  if (id >= vocab) {
    if (threadIdx.x == 0 && err) atomicOr(err, kErrBadToken);
    id = 0;
  }
  for (uint32_t i = threadIdx.x; i < d; i += blockDim.x)
    x[(size_t)t * d + i] = dequant_native_elem(type, emb, (uint64_t)id * d + i);
}

__device__ float block_sum(float v, float *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  const uint32_t w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float s = 0.0f;
  for (uint32_t i = 0; i < nw; ++i) s += red[i];
  __syncthreads();
  return s;
}

constexpr float kHalfMax = 65504.0f;

__global__ void k_norm_rows_h(const float *x, const float *w, float eps, uint32_t d, __half *out, uint32_t *err) {
  pdl_enter();
  __shared__ float red[32];
  const float *r = x + (size_t)blockIdx.x * d;
  constexpr uint32_t kV = 8;  // float4 of the row per thread held in registers (rows up to 8192 wide)
  if (d % (4 * blockDim.x) == 0 && d <= 4 * kV * blockDim.x) {
    // the thread's slice of the row and of the norm weights in one round trip
    const uint32_t nv = d / (4 * blockDim.x);
    float4 xv[kV], wv[kV];
#pragma unroll
    for (uint32_t j = 0; j < kV; ++j)
      if (j < nv) {
        xv[j] = __ldcg(reinterpret_cast<const float4 *>(r) + j * blockDim.x + threadIdx.x);
        wv[j] = __ldg(reinterpret_cast<const float4 *>(w) + j * blockDim.x + threadIdx.x);
      }
    float s = 0.0f;
#pragma unroll
    for (uint32_t j = 0; j < kV; ++j)
      if (j < nv) {
        s = fmaf(xv[j].x, xv[j].x, s);
        s = fmaf(xv[j].y, xv[j].y, s);
        s = fmaf(xv[j].z, xv[j].z, s);
        s = fmaf(xv[j].w, xv[j].w, s);
      }
    s = block_sum(s, red);
    const float inv = 1.0f / sqrtf(s / (float)d + eps);
    bool bad = false;
#pragma unroll
    for (uint32_t j = 0; j < kV; ++j)
      if (j < nv) {
        const float a = __fmul_rn(__fmul_rn(xv[j].x, inv), wv[j].x), b = __fmul_rn(__fmul_rn(xv[j].y, inv), wv[j].y);
        const float c = __fmul_rn(__fmul_rn(xv[j].z, inv), wv[j].z), e = __fmul_rn(__fmul_rn(xv[j].w, inv), wv[j].w);
        bad |= !(fabsf(a) <= kHalfMax) || !(fabsf(b) <= kHalfMax) || !(fabsf(c) <= kHalfMax) || !(fabsf(e) <= kHalfMax);
        __half2 *o = reinterpret_cast<__half2 *>(out + (size_t)blockIdx.x * d) + 2 * (j * blockDim.x + threadIdx.x);
        o[0] = __floats2half2_rn(a, b);
        o[1] = __floats2half2_rn(c, e);
      }
    if (bad && err) atomicOr(err, kErrRange);
    return;
  }
  float s = 0.0f;
  for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) s = fmaf(r[i], r[i], s);
  s = block_sum(s, red);
  const float inv = 1.0f / sqrtf(s / (float)d + eps);
  bool bad = false;
  for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) {
    const float v = __fmul_rn(__fmul_rn(r[i], inv), w[i]);
    bad |= !(fabsf(v) <= kHalfMax);
    out[(size_t)blockIdx.x * d + i] = __float2half_rn(v);
  }
  if (bad && err) atomicOr(err, kErrRange);
}

// one CTA per token; rows of QKV: [q (Hq*hd) | k (Hkv*hd) | v (Hkv*hd)]
__global__ void k_rope_kv_rows(const float *qkv, uint32_t T, uint32_t Hq, uint32_t Hkv, uint32_t hd, const float *rope,
                               uint32_t rope_max, uint32_t pos0, uint32_t len0, KvView kv, uint32_t seq, uint32_t layer,
                               __half *qh, uint32_t *err) {
  pdl_enter();
  const uint32_t t = blockIdx.x, half = hd / 2, qd = Hq * hd, kd = Hkv * hd;
  const float *row = qkv + (size_t)t * (qd + 2 * kd);
  const uint32_t pos = pos0 + t, slot = len0 + t;
  if (pos >= rope_max || slot / 16 >= kv.max_pages) {
    if (threadIdx.x == 0 && err) atomicOr(err, kErrContext);
    return;
  }
  const float *cs = rope + (size_t)pos * hd;
  const uint32_t page = kv.page_table[seq * kv.max_pages + slot / 16];
  const uint64_t lbase = (uint64_t)layer * kv.layer_stride;
  for (uint32_t j = threadIdx.x; j < qd + 2 * kd; j += blockDim.x) {
    float v = row[j];
    const bool is_q = j < qd, is_k = !is_q && j < qd + kd;
    if (is_q || is_k) {
      const uint32_t base = is_q ? 0 : qd, dd = (j - base) % hd, hb = j - dd;
      const float cth = cs[2 * (dd % half)], sth = cs[2 * (dd % half) + 1];
      const float pv = dd < half ? row[hb + dd + half] : row[hb + dd - half];
      v = dd < half ? __fsub_rn(__fmul_rn(v, cth), __fmul_rn(pv, sth)) : __fadd_rn(__fmul_rn(pv, sth), __fmul_rn(v, cth));
    }
    if (is_q) {
      qh[(size_t)t * qd + j] = __float2half_rn(v);
    } else {
      const uint32_t kc = is_k ? j - qd : j - qd - kd;
      const uint64_t idx = lbase + kv_index(page, is_k ? 0 : 1, kc / hd, slot % 16, kc % hd, kv.n_kv, hd);
      if (kv.f16) reinterpret_cast<__half *>(kv.base)[idx] = __float2half_rn(v);
      else reinterpret_cast<float *>(kv.base)[idx] = v;
    }
  }
}

// The same with four elements per work unit (hd % 4 == 0): a q or k head's
// unit is dims (d, d + 1) and their rotation partners (d + hd/2, d + hd/2 + 1)
// for d even < hd/2 (one float4 of cos/sin), a v unit four consecutive dims;
// paired loads and stores, the same per-element rounding.
__global__ void k_rope_kv_rows4(const float *qkv, uint32_t T, uint32_t Hq, uint32_t Hkv, uint32_t hd,
                                const float *rope, uint32_t rope_max, uint32_t pos0, uint32_t len0, KvView kv,
                                uint32_t seq, uint32_t layer, __half *qh, uint32_t *err) {
  pdl_enter();
  const uint32_t t = blockIdx.x, half = hd / 2, qd = Hq * hd, kd = Hkv * hd;
  const float *row = qkv + (size_t)t * (qd + 2 * kd);
  const uint32_t pos = pos0 + t, slot = len0 + t;
  if (pos >= rope_max || slot / 16 >= kv.max_pages) {
    if (threadIdx.x == 0 && err) atomicOr(err, kErrContext);
    return;
  }
  const float *cs = rope + (size_t)pos * hd;
  const uint32_t page = kv.page_table[seq * kv.max_pages + slot / 16];
  const uint64_t lbase = (uint64_t)layer * kv.layer_stride;
  const uint32_t upr = half / 2, n_rot = (Hq + Hkv) * upr, n_units = n_rot + kd / 4;
  auto put2 = [&](uint64_t idx, float a, float b) {  // two consecutive cache elements
    if (kv.f16) *reinterpret_cast<__half2 *>(reinterpret_cast<__half *>(kv.base) + idx) = __floats2half2_rn(a, b);
    else *reinterpret_cast<float2 *>(reinterpret_cast<float *>(kv.base) + idx) = make_float2(a, b);
  };
  for (uint32_t u = threadIdx.x; u < n_units; u += blockDim.x) {
    if (u < n_rot) {
      const uint32_t head = u / upr, dd = 2 * (u % upr), hb = head * hd;
      const float2 x = *reinterpret_cast<const float2 *>(row + hb + dd);
      const float2 y = *reinterpret_cast<const float2 *>(row + hb + dd + half);
      const float4 c = *reinterpret_cast<const float4 *>(cs + 2 * dd);  // cos, sin of dd and dd + 1
      const float a0 = __fsub_rn(__fmul_rn(x.x, c.x), __fmul_rn(y.x, c.y));
      const float a1 = __fsub_rn(__fmul_rn(x.y, c.z), __fmul_rn(y.y, c.w));
      const float b0 = __fadd_rn(__fmul_rn(x.x, c.y), __fmul_rn(y.x, c.x));
      const float b1 = __fadd_rn(__fmul_rn(x.y, c.w), __fmul_rn(y.y, c.z));
      if (head < Hq) {
        __half *q = qh + (size_t)t * qd + hb + dd;
        *reinterpret_cast<__half2 *>(q) = __floats2half2_rn(a0, a1);
        *reinterpret_cast<__half2 *>(q + half) = __floats2half2_rn(b0, b1);
      } else {
        const uint64_t idx = lbase + kv_index(page, 0, head - Hq, slot % 16, dd, kv.n_kv, hd);
        put2(idx, a0, a1);
        put2(idx + half, b0, b1);
      }
    } else {
      const uint32_t kc = 4 * (u - n_rot);
      const float4 v = *reinterpret_cast<const float4 *>(row + qd + kd + kc);
      const uint64_t idx = lbase + kv_index(page, 1, kc / hd, slot % 16, kc % hd, kv.n_kv, hd);
      put2(idx, v.x, v.y);
      put2(idx + 2, v.z, v.w);
    }
  }
}

// ---- causal flash attention (mma.sync m16n8k16 f16, f32 accumulation) ----
constexpr uint32_t kAQ = 64, kAK = 64;  // query rows and cache slots per tile

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&h);
}
// byte offset of 16-byte chunk c of row r in a tile of rows of `rb` bytes
// (chunks XOR-swizzled by row so 8 consecutive rows hit distinct banks)
__device__ __forceinline__ uint32_t sw_off(uint32_t r, uint32_t c, uint32_t rb) { return r * rb + ((c ^ (r & 7)) << 4); }

// stage cache slots [s0, s0 + 64) of (kv head, K or V) into a tile of rows of
// HD f16; slots >= s_end read as zero
template <uint32_t HD, bool F16>
__device__ __forceinline__ void load_kv_tile(const KvView &kv, uint64_t lbase, const uint32_t *pt, uint32_t kvh,
                                             int is_v, uint32_t s0, uint32_t s_end, uint32_t tile) {
  constexpr uint32_t CH = HD / 8;  // 16-byte chunks per row
  for (uint32_t i = threadIdx.x; i < kAK * CH; i += blockDim.x) {
    const uint32_t r = i / CH, c = i % CH, s = s0 + r;
    const uint32_t dst = tile + sw_off(r, c, HD * 2);
    if (s >= s_end) {
      asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(dst), "r"(0u) : "memory");
      continue;
    }
    const uint64_t idx = lbase + kv_index(pt[s / 16], is_v, kvh, s % 16, 8 * c, kv.n_kv, HD);
    if (F16) {
      const __half *src = reinterpret_cast<const __half *>(kv.base) + idx;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
    } else {
      const float4 *src = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(kv.base) + idx);
      const float4 a = __ldcg(src), b = __ldcg(src + 1);
      asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(pack_h2(a.x, a.y)), "r"(pack_h2(a.z, a.w)),
                   "r"(pack_h2(b.x, b.y)), "r"(pack_h2(b.z, b.w))
                   : "memory");
    }
  }
}

// The same for an f16 cache, K and V at once, 128 threads, s0 a multiple
// of 64 (four whole pages): thread i copies chunk i % 16 of rows i / 16 + 8j
// (j = 0..7: page j / 2, slot i / 16 + 8 (j & 1)); the row's swizzle term
// is the thread's own (rows differ by multiples of 8), so the destination
// is a per-thread base plus 2048 j.
template <uint32_t HD>
__device__ __forceinline__ void load_kv_tiles_f16(const KvView &kv, uint64_t lbase, const uint32_t *pt, uint32_t kvh,
                                                  uint32_t s0, uint32_t s_end, uint32_t ktile, uint32_t vtile) {
  static_assert(HD == 128 && kAK == 64, "64 rows of 16 chunks over 128 threads");
  const uint32_t c = threadIdx.x & 15, r0 = threadIdx.x >> 4;
  const __half *base = reinterpret_cast<const __half *>(kv.base) + lbase;
  const uint64_t vofs = (uint64_t)kv.n_kv * 16 * HD;  // V block of (page, kv head) after the K blocks
  const uint32_t dst0 = r0 * HD * 2 + ((c ^ r0) << 4);
  const bool full = s0 + kAK <= s_end;
#pragma unroll
  for (uint32_t q = 0; q < 4; ++q) {
    if (!(s0 + 16 * q < s_end)) {  // pages past the slots this tile reads are not looked up
#pragma unroll
      for (uint32_t jj = 0; jj < 2; ++jj) {
        const uint32_t off = dst0 + (2 * q + jj) * 8 * HD * 2;
        asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(ktile + off), "r"(0u) : "memory");
        asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(vtile + off), "r"(0u) : "memory");
      }
      continue;
    }
    const __half *src0 = base + kv_index(pt[s0 / 16 + q], 0, kvh, r0, 8 * c, kv.n_kv, HD);
#pragma unroll
    for (uint32_t jj = 0; jj < 2; ++jj) {
      const uint32_t off = dst0 + (2 * q + jj) * 8 * HD * 2;
      const __half *src = src0 + 8 * jj * HD;
      if (full || s0 + 16 * q + 8 * jj + r0 < s_end) {
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(ktile + off), "l"(src) : "memory");
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(vtile + off), "l"(src + vofs) : "memory");
      } else {
        asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(ktile + off), "r"(0u) : "memory");
        asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(vtile + off), "r"(0u) : "memory");
      }
    }
  }
}

// grid (query tiles, q heads); 4 warps x 16 query rows
template <uint32_t HD, bool F16>
__global__ void __launch_bounds__(128) k_attn_causal(const __half *qh, uint32_t T, uint32_t Hq, uint32_t Hkv,
                                                     uint32_t len0, KvView kv, uint32_t seq, uint32_t layer,
                                                     float scale_log2, __half *out) {
  pdl_enter();
  extern __shared__ __align__(128) uint8_t asm_raw[];
  constexpr uint32_t RB = HD * 2, KT = HD / 16, NT = kAK / 8, OT = HD / 8;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const uint32_t h = blockIdx.y, kvh = h / (Hq / Hkv), t0 = blockIdx.x * kAQ;
  const uint32_t ks_tile = smem_u32(asm_raw), vs_tile = ks_tile + kAK * RB;
  const uint64_t lbase = (uint64_t)layer * kv.layer_stride;
  const uint32_t *pt = kv.page_table + (size_t)seq * kv.max_pages;
  const uint32_t last_t = min(T, t0 + kAQ) - 1, s_end = len0 + last_t + 1;  // slots this tile may read
  // Q fragments of this warp's 16 rows (rows >= T read as zero)
  uint32_t qa[KT][4];
  {
    const uint32_t r0 = t0 + 16 * warp + g, r1 = r0 + 8;
#pragma unroll
    for (uint32_t kt = 0; kt < KT; ++kt) {
      const uint32_t d0 = 16 * kt + 2 * c;
      auto ld = [&](uint32_t r, uint32_t d) -> uint32_t {
        return r < T ? *reinterpret_cast<const uint32_t *>(qh + (size_t)r * Hq * HD + h * HD + d) : 0u;
      };
      qa[kt][0] = ld(r0, d0);
      qa[kt][1] = ld(r1, d0);
      qa[kt][2] = ld(r0, d0 + 8);
      qa[kt][3] = ld(r1, d0 + 8);
    }
  }
  float o[OT][4];
#pragma unroll
  for (uint32_t j = 0; j < OT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  const uint32_t q0 = t0 + 16 * warp + g, q1 = q0 + 8;  // query tokens of this lane's rows
  for (uint32_t s0 = 0; s0 < s_end; s0 += kAK) {
    if constexpr (F16 && HD == 128) {
      load_kv_tiles_f16<HD>(kv, lbase, pt, kvh, s0, s_end, ks_tile, vs_tile);
    } else {
      load_kv_tile<HD, F16>(kv, lbase, pt, kvh, 0, s0, s_end, ks_tile);
      load_kv_tile<HD, F16>(kv, lbase, pt, kvh, 1, s0, s_end, vs_tile);
    }
    if (F16) asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    // S = Q K^T for 16 rows x 64 slots
    float s[NT][4];
#pragma unroll
    for (uint32_t j = 0; j < NT; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (uint32_t kt = 0; kt < KT; ++kt) {
#pragma unroll
      for (uint32_t j = 0; j < NT; j += 2) {
        // matrices: (slots 8j.., dims 16kt), (8j.., 16kt+8), (8j+8.., 16kt), (8j+8.., 16kt+8)
        const uint32_t mi = lane >> 3, r = 8 * j + 8 * (mi >> 1) + (lane & 7), ch = 2 * kt + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(ks_tile + sw_off(r, ch, RB), b0, b1, b2, b3);
        mma_f16(s[j], qa[kt][0], qa[kt][1], qa[kt][2], qa[kt][3], b0, b1);
        mma_f16(s[j + 1], qa[kt][0], qa[kt][1], qa[kt][2], qa[kt][3], b2, b3);
      }
    }
    // causal mask, online softmax (base 2)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (uint32_t j = 0; j < NT; ++j) {
      const uint32_t sl = s0 + 8 * j + 2 * c;
#pragma unroll
      for (uint32_t e = 0; e < 2; ++e) {
        s[j][e] = (sl + e <= len0 + q0 && sl + e < s_end) ? s[j][e] * scale_log2 : -INFINITY;
        s[j][2 + e] = (sl + e <= len0 + q1 && sl + e < s_end) ? s[j][2 + e] * scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, s[j][e]);
        mx1 = fmaxf(mx1, s[j][2 + e]);
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, off));
    }
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float a0 = n0 == -INFINITY ? 1.0f : exp2f(m0 - n0), a1 = n1 == -INFINITY ? 1.0f : exp2f(m1 - n1);
    float ls0 = 0.0f, ls1 = 0.0f;
#pragma unroll
    for (uint32_t j = 0; j < NT; ++j) {
#pragma unroll
      for (uint32_t e = 0; e < 2; ++e) {
        s[j][e] = n0 == -INFINITY ? 0.0f : exp2f(s[j][e] - n0);
        s[j][2 + e] = n1 == -INFINITY ? 0.0f : exp2f(s[j][2 + e] - n1);
        ls0 += s[j][e];
        ls1 += s[j][2 + e];
      }
    }
    l0 = fmaf(l0, a0, ls0);
    l1 = fmaf(l1, a1, ls1);
    m0 = n0;
    m1 = n1;
#pragma unroll
    for (uint32_t j = 0; j < OT; ++j) {
      o[j][0] *= a0;
      o[j][1] *= a0;
      o[j][2] *= a1;
      o[j][3] *= a1;
    }
    // O += P V: P (16 x 64) as A fragments, V rows of slots via transposed ldmatrix
#pragma unroll
    for (uint32_t kt = 0; kt < kAK / 16; ++kt) {
      const uint32_t pa0 = pack_h2(s[2 * kt][0], s[2 * kt][1]), pa1 = pack_h2(s[2 * kt][2], s[2 * kt][3]);
      const uint32_t pa2 = pack_h2(s[2 * kt + 1][0], s[2 * kt + 1][1]), pa3 = pack_h2(s[2 * kt + 1][2], s[2 * kt + 1][3]);
#pragma unroll
      for (uint32_t j = 0; j < OT; j += 2) {
        // matrices: (slots 16kt.., dims 8j), (16kt+8.., 8j), (16kt.., 8j+8), (16kt+8.., 8j+8)
        const uint32_t mi = lane >> 3, r = 16 * kt + 8 * (mi & 1) + (lane & 7), ch = j + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vs_tile + sw_off(r, ch, RB), b0, b1, b2, b3);
        mma_f16(o[j], pa0, pa1, pa2, pa3, b0, b1);
        mma_f16(o[j + 1], pa0, pa1, pa2, pa3, b2, b3);
      }
    }
    __syncthreads();
  }
  // rows: lane sums across the 4 lanes of a row, then O / l
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, off);
    l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, off);
  }
  const float i0 = l0 > 0.0f ? 1.0f / l0 : 0.0f, i1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
#pragma unroll
  for (uint32_t j = 0; j < OT; ++j) {
    const uint32_t d = 8 * j + 2 * c;
    if (q0 < T) *reinterpret_cast<__half2 *>(out + (size_t)q0 * Hq * HD + h * HD + d) = __floats2half2_rn(o[j][0] * i0, o[j][1] * i0);
    if (q1 < T) *reinterpret_cast<__half2 *>(out + (size_t)q1 * Hq * HD + h * HD + d) = __floats2half2_rn(o[j][2] * i1, o[j][3] * i1);
  }
}

// ---- batched decode attention on the tensor cores: one query token per row,
// the REP query heads of a kv head as the MMA rows (padded to 16); grid
// (splits, kv heads, rows), 4 warps each streaming 32-position K/V tiles of
// the split (cp.async into private swizzled tiles), S = Q K^T and O += P V by
// mma.sync, online softmax in base 2; warps merge in shared memory, the last
// split of a (row, kv head) combines all splits in a fixed order ----
constexpr uint32_t kDT = 32;

template <uint32_t HD, bool F16>
__device__ __forceinline__ void stage_rows(const KvView &kv, uint64_t lbase, const uint32_t *pt, uint32_t kvh,
                                           int is_v, uint32_t s0, uint32_t s_end, uint32_t tile, uint32_t lane) {
  constexpr uint32_t CH = HD / 8;
  for (uint32_t i = lane; i < kDT * CH; i += 32) {
    const uint32_t r = i / CH, c = i % CH, s = s0 + r;
    const uint32_t dst = tile + sw_off(r, c, HD * 2);
    if (s >= s_end) {
      asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(dst), "r"(0u) : "memory");
      continue;
    }
    const uint64_t idx = lbase + kv_index(pt[s / 16], is_v, kvh, s % 16, 8 * c, kv.n_kv, HD);
    if (F16) {
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(reinterpret_cast<const __half *>(kv.base) + idx)
                   : "memory");
    } else {
      const float4 *src = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(kv.base) + idx);
      const float4 a = __ldcg(src), b = __ldcg(src + 1);
      asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(pack_h2(a.x, a.y)), "r"(pack_h2(a.z, a.w)),
                   "r"(pack_h2(b.x, b.y)), "r"(pack_h2(b.z, b.w))
                   : "memory");
    }
  }
}

// The same for an f16 cache, K and V at once, s0 a multiple of 32: the tile
// is two whole pages, so lane l's chunks are (row 2j + l / 16, chunk l % 16)
// for j = 0..15, in page j / 8 at a fixed offset from the lane's base, and
// the swizzled destination is a per-lane base plus a constant (row bit 0 is
// the lane's, rows differ by multiples of 2 in the XOR).
template <uint32_t HD>
__device__ __forceinline__ void stage_kv_f16(const KvView &kv, uint64_t lbase, const uint32_t *pt, uint32_t kvh,
                                             uint32_t s0, uint32_t s_end, uint32_t ktile, uint32_t vtile,
                                             uint32_t lane) {
  static_assert(HD == 128, "two rows of 16 chunks per warp-wide copy");
  const uint32_t c = lane & 15, r0 = lane >> 4;
  const __half *base = reinterpret_cast<const __half *>(kv.base) + lbase;
  const uint64_t vofs = (uint64_t)kv.n_kv * 16 * HD;  // V block of (page, kv head) after the K blocks
  const __half *kp[2];
#pragma unroll
  for (uint32_t q = 0; q < 2; ++q)  // pages past the sequence's end are not read
    kp[q] = s0 + 16 * q < s_end ? base + kv_index(pt[s0 / 16 + q], 0, kvh, r0, 8 * c, kv.n_kv, HD) : base;
  uint32_t xo[4];
#pragma unroll
  for (uint32_t m = 0; m < 4; ++m) xo[m] = ((c ^ r0) ^ (2 * m)) << 4;
  const uint32_t row0 = r0 * HD * 2;
  const bool full = s0 + kDT <= s_end;
#pragma unroll
  for (uint32_t j = 0; j < 16; ++j) {
    const uint32_t off = row0 + 2 * j * HD * 2 + xo[j & 3];
    const __half *src = kp[j >> 3] + 2 * (j & 7) * HD;
    if (full || s0 + 2 * j + r0 < s_end) {
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(ktile + off), "l"(src) : "memory");
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(vtile + off), "l"(src + vofs) : "memory");
    } else {
      asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(ktile + off), "r"(0u) : "memory");
      asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(vtile + off), "r"(0u) : "memory");
    }
  }
}

template <uint32_t HD, bool F16, uint32_t REP>
__global__ void __launch_bounds__(128, 3) k_attn_decode_rows(const AttnParams p, float scale_log2) {
  pdl_enter();
  extern __shared__ __align__(128) uint8_t dsm[];
  constexpr uint32_t RB = HD * 2, KT = HD / 16, NT = kDT / 8, OT = HD / 8, W = 2 + HD;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
  const uint32_t split = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z, KVH = p.kv.n_kv, H = p.n_heads;
  const uint32_t T = p.row_states[row].len + 1, seq = p.row_seq0 + row;
  uint32_t Ls = (T + p.splits - 1) / p.splits;
  Ls = (Ls + kDT - 1) / kDT * kDT;
  const uint32_t t0 = min(T, split * Ls), t1 = min(T, t0 + Ls);
  const uint32_t ktile = smem_u32(dsm) + warp * 2 * kDT * RB, vtile = ktile + kDT * RB;
  const uint64_t lbase = (uint64_t)p.layer * p.kv.layer_stride;
  const uint32_t *pt = p.kv.page_table + (size_t)seq * p.kv.max_pages;
  // Q fragments: MMA rows = the query heads of this kv head (rows >= REP are zero)
  const float *qr = p.q + (size_t)row * H * HD + (size_t)kvh * REP * HD;
  uint32_t qa[KT][4];
#pragma unroll
  for (uint32_t kt = 0; kt < KT; ++kt) {
    const uint32_t d0 = 16 * kt + 2 * c;
    auto ld = [&](uint32_t r, uint32_t d) -> uint32_t {
      return r < REP ? pack_h2(qr[r * HD + d], qr[r * HD + d + 1]) : 0u;
    };
    qa[kt][0] = ld(g, d0);
    qa[kt][1] = ld(g + 8, d0);
    qa[kt][2] = ld(g, d0 + 8);
    qa[kt][3] = ld(g + 8, d0 + 8);
  }
  float o[OT][4];
#pragma unroll
  for (uint32_t j = 0; j < OT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  for (uint32_t s0 = t0 + warp * kDT; s0 < t1; s0 += 4 * kDT) {
    if constexpr (F16 && HD == 128) {
      stage_kv_f16<HD>(p.kv, lbase, pt, kvh, s0, t1, ktile, vtile, lane);
    } else {
      stage_rows<HD, F16>(p.kv, lbase, pt, kvh, 0, s0, t1, ktile, lane);
      stage_rows<HD, F16>(p.kv, lbase, pt, kvh, 1, s0, t1, vtile, lane);
    }
    if (F16) asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
    float s[NT][4];
#pragma unroll
    for (uint32_t j = 0; j < NT; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (uint32_t kt = 0; kt < KT; ++kt)
#pragma unroll
      for (uint32_t j = 0; j < NT; j += 2) {
        const uint32_t mi = lane >> 3, r = 8 * j + 8 * (mi >> 1) + (lane & 7), ch = 2 * kt + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(ktile + sw_off(r, ch, RB), b0, b1, b2, b3);
        mma_f16(s[j], qa[kt][0], qa[kt][1], qa[kt][2], qa[kt][3], b0, b1);
        mma_f16(s[j + 1], qa[kt][0], qa[kt][1], qa[kt][2], qa[kt][3], b2, b3);
      }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (uint32_t j = 0; j < NT; ++j)
#pragma unroll
      for (uint32_t e = 0; e < 2; ++e) {
        const bool ok = s0 + 8 * j + 2 * c + e < t1;
        s[j][e] = ok ? s[j][e] * scale_log2 : -INFINITY;
        s[j][2 + e] = ok ? s[j][2 + e] * scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, s[j][e]);
        mx1 = fmaxf(mx1, s[j][2 + e]);
      }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, off));
    }
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float a0 = n0 == -INFINITY ? 1.0f : exp2f(m0 - n0), a1 = n1 == -INFINITY ? 1.0f : exp2f(m1 - n1);
    float ls0 = 0.0f, ls1 = 0.0f;
#pragma unroll
    for (uint32_t j = 0; j < NT; ++j)
#pragma unroll
      for (uint32_t e = 0; e < 2; ++e) {
        s[j][e] = n0 == -INFINITY ? 0.0f : exp2f(s[j][e] - n0);
        s[j][2 + e] = n1 == -INFINITY ? 0.0f : exp2f(s[j][2 + e] - n1);
        ls0 += s[j][e];
        ls1 += s[j][2 + e];
      }
    l0 = fmaf(l0, a0, ls0);
    l1 = fmaf(l1, a1, ls1);
    m0 = n0;
    m1 = n1;
#pragma unroll
    for (uint32_t j = 0; j < OT; ++j) {
      o[j][0] *= a0;
      o[j][1] *= a0;
      o[j][2] *= a1;
      o[j][3] *= a1;
    }
#pragma unroll
    for (uint32_t kt = 0; kt < kDT / 16; ++kt) {
      const uint32_t pa0 = pack_h2(s[2 * kt][0], s[2 * kt][1]), pa1 = pack_h2(s[2 * kt][2], s[2 * kt][3]);
      const uint32_t pa2 = pack_h2(s[2 * kt + 1][0], s[2 * kt + 1][1]), pa3 = pack_h2(s[2 * kt + 1][2], s[2 * kt + 1][3]);
#pragma unroll
      for (uint32_t j = 0; j < OT; j += 2) {
        const uint32_t mi = lane >> 3, r = 16 * kt + 8 * (mi & 1) + (lane & 7), ch = j + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vtile + sw_off(r, ch, RB), b0, b1, b2, b3);
        mma_f16(o[j], pa0, pa1, pa2, pa3, b0, b1);
        mma_f16(o[j + 1], pa0, pa1, pa2, pa3, b2, b3);
      }
    }
    __syncwarp();  // the next tile overwrites this warp's K/V tiles
  }
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, off);
    l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, off);
  }
  // merge the 4 warps (the tile memory becomes scratch [warp][16 rows][W])
  __syncthreads();
  float *scr = reinterpret_cast<float *>(dsm);
  float *sw = scr + (size_t)warp * 16 * W;
  if (c == 0) {
    sw[g * W] = m0;
    sw[g * W + 1] = l0;
    sw[(g + 8) * W] = m1;
    sw[(g + 8) * W + 1] = l1;
  }
#pragma unroll
  for (uint32_t j = 0; j < OT; ++j)
#pragma unroll
    for (uint32_t e = 0; e < 2; ++e) {
      sw[g * W + 2 + 8 * j + 2 * c + e] = o[j][e];
      sw[(g + 8) * W + 2 + 8 * j + 2 * c + e] = o[j][2 + e];
    }
  __syncthreads();
  float *part = p.part + (size_t)row * H * p.splits * W;
  for (uint32_t idx = tid; idx < REP * W; idx += 128) {
    const uint32_t r = idx / W, cc = idx % W;
    float M = -INFINITY;
    for (uint32_t w = 0; w < 4; ++w) M = fmaxf(M, scr[(w * 16 + r) * W]);
    float v = M;
    if (cc) {
      v = 0.0f;
      for (uint32_t w = 0; w < 4; ++w) {
        const float mw = scr[(w * 16 + r) * W];
        if (mw != -INFINITY) v = fmaf(scr[(w * 16 + r) * W + cc], exp2f(mw - M), v);
      }
    }
    part[((kvh * REP + r) * p.splits + split) * W + cc] = v;
  }
  __threadfence();
  __syncthreads();
  __shared__ uint32_t last;
  uint32_t *cnt = p.counters + (size_t)row * KVH + kvh;
  if (tid == 0) last = atomicAdd(cnt, 1u) + 1 == p.splits ? 1u : 0u;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // combine the splits of (row, kv head) in split order
  for (uint32_t idx = tid; idx < REP * HD; idx += 128) {
    const uint32_t r = idx / HD, d = idx % HD;
    const float *P = part + (size_t)(kvh * REP + r) * p.splits * W;
    float M = -INFINITY;
    for (uint32_t sp = 0; sp < p.splits; ++sp) M = fmaxf(M, __ldcg(P + sp * W));
    float L = 0.0f, acc = 0.0f;
    for (uint32_t sp = 0; sp < p.splits; ++sp) {
      const float ms = __ldcg(P + sp * W);
      if (ms == -INFINITY) continue;
      const float e = exp2f(ms - M);
      L = fmaf(__ldcg(P + sp * W + 1), e, L);
      acc = fmaf(__ldcg(P + sp * W + 2 + d), e, acc);
    }
    const float y = L > 0.0f ? acc / L : 0.0f;
    const size_t o = (size_t)row * H * HD + (size_t)(kvh * REP + r) * HD + d;
    if (p.out_h) {  // straight to the f16 operand of the o GEMM
      if (!(fabsf(y) <= kHalfMax) && p.err) atomicOr(p.err, kErrRange);
      reinterpret_cast<__half *>(p.out_h)[o] = __float2half_rn(y);
    } else {
      p.out[o] = y;
    }
  }
  if (tid == 0) *cnt = 0u;
}

// gate/up launch space: chunk c (width w_c) holds gate f in [c*CW/2, +w_c/2)
// at c*CW + local, then the same up columns
__global__ void k_swiglu_rows(const float *gu, uint32_t F, uint32_t CW, __half *h, uint32_t *err) {
  pdl_enter();
  const uint32_t t = blockIdx.y, f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= F) return;
  const uint32_t c = f / (CW / 2), local = f - c * (CW / 2), wc = min(CW, 2 * F - c * CW);
  const float *row = gu + (size_t)t * 2 * F;
  const float gv = row[c * CW + local], uv = row[c * CW + wc / 2 + local];
  const float v = gv * (1.0f / (1.0f + expf(-gv))) * uv;
  if (!(fabsf(v) <= kHalfMax) && err) atomicOr(err, kErrRange);
  h[(size_t)t * F + f] = __float2half_rn(v);
}

// The same, four consecutive columns per thread (F % 4 == 0, CW % 32 == 0:
// the four stay inside one chunk half and the loads are float4-aligned),
// streaming loads, one 8-byte store; the same per-element arithmetic.
__global__ void k_swiglu_rows4(const float *gu, uint32_t F, uint32_t CW, __half *h, uint32_t *err) {
  pdl_enter();
  const uint32_t t = blockIdx.y, f = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (f >= F) return;
  const uint32_t hw = CW / 2, c = f / hw, local = f - c * hw, wc = min(CW, 2 * F - c * CW);
  const float *row = gu + (size_t)t * 2 * F + (size_t)c * CW + local;
  const float4 g4 = __ldcs(reinterpret_cast<const float4 *>(row));
  const float4 u4 = __ldcs(reinterpret_cast<const float4 *>(row + wc / 2));
  const float gv[4] = {g4.x, g4.y, g4.z, g4.w}, uv[4] = {u4.x, u4.y, u4.z, u4.w};
  float v[4];
  bool bad = false;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    v[e] = gv[e] * (1.0f / (1.0f + expf(-gv[e]))) * uv[e];
    bad |= !(fabsf(v[e]) <= kHalfMax);
  }
  if (bad && err) atomicOr(err, kErrRange);
  const __half2 lo = __floats2half2_rn(v[0], v[1]), hi = __floats2half2_rn(v[2], v[3]);
  uint2 o;
  o.x = *reinterpret_cast<const uint32_t *>(&lo);
  o.y = *reinterpret_cast<const uint32_t *>(&hi);
  *reinterpret_cast<uint2 *>(h + (size_t)t * F + f) = o;
}

// last token's row -> x, its sum of squares -> ssq[0] (the rest zero)
__global__ void k_last_row(const float *X, uint32_t row, uint32_t d, float *x, float *ssq, uint32_t n_ssq) {
  pdl_enter();
  __shared__ float red[32];
  float s = 0.0f;
  for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) {
    const float v = X[(size_t)row * d + i];
    x[i] = v;
    s = fmaf(v, v, s);
  }
  s = block_sum(s, red);
  for (uint32_t i = threadIdx.x; i < n_ssq; i += blockDim.x) ssq[i] = i == 0 ? s : 0.0f;
}

// ---- batched decode: row r is cache sequence seq0 + r at its own position ----
// The same with the four-element units of k_rope_kv_rows4 (hd % 4 == 0),
// grid (rows, unit blocks): one unit per thread, q kept in f32.
__global__ void k_rope_kv_batch4(const float *qkv, uint32_t Hq, uint32_t Hkv, uint32_t hd, const float *rope,
                                 uint32_t rope_max, const SeqState *st, KvView kv, uint32_t seq0, uint32_t layer,
                                 float *qf, uint32_t *err) {
  pdl_enter();
  const uint32_t r = blockIdx.x, half = hd / 2, qd = Hq * hd, kd = Hkv * hd;
  const uint32_t upr = half / 2, n_rot = (Hq + Hkv) * upr, n_units = n_rot + kd / 4;
  const uint32_t u = blockIdx.y * blockDim.x + threadIdx.x;
  const float *row = qkv + (size_t)r * (qd + 2 * kd);
  const uint32_t pos = st[r].pos, slot = st[r].len;
  if (pos >= rope_max || slot / 16 >= kv.max_pages) {
    if (u == 0 && err) atomicOr(err, kErrContext);
    return;
  }
  if (u >= n_units) return;
  const uint32_t page = kv.page_table[(seq0 + r) * kv.max_pages + slot / 16];
  const uint64_t lbase = (uint64_t)layer * kv.layer_stride;
  auto put2 = [&](uint64_t idx, float a, float b) {  // two consecutive cache elements
    if (kv.f16) *reinterpret_cast<__half2 *>(reinterpret_cast<__half *>(kv.base) + idx) = __floats2half2_rn(a, b);
    else *reinterpret_cast<float2 *>(reinterpret_cast<float *>(kv.base) + idx) = make_float2(a, b);
  };
  if (u < n_rot) {
    const uint32_t head = u / upr, dd = 2 * (u % upr), hb = head * hd;
    const float2 x = *reinterpret_cast<const float2 *>(row + hb + dd);
    const float2 y = *reinterpret_cast<const float2 *>(row + hb + dd + half);
    const float4 c = *reinterpret_cast<const float4 *>(rope + (size_t)pos * hd + 2 * dd);  // cos, sin of dd, dd + 1
    const float a0 = __fsub_rn(__fmul_rn(x.x, c.x), __fmul_rn(y.x, c.y));
    const float a1 = __fsub_rn(__fmul_rn(x.y, c.z), __fmul_rn(y.y, c.w));
    const float b0 = __fadd_rn(__fmul_rn(x.x, c.y), __fmul_rn(y.x, c.x));
    const float b1 = __fadd_rn(__fmul_rn(x.y, c.w), __fmul_rn(y.y, c.z));
    if (head < Hq) {
      float *q = qf + (size_t)r * qd + hb + dd;
      *reinterpret_cast<float2 *>(q) = make_float2(a0, a1);
      *reinterpret_cast<float2 *>(q + half) = make_float2(b0, b1);
    } else {
      const uint64_t idx = lbase + kv_index(page, 0, head - Hq, slot % 16, dd, kv.n_kv, hd);
      put2(idx, a0, a1);
      put2(idx + half, b0, b1);
    }
  } else {
    const uint32_t kc = 4 * (u - n_rot);
    const float4 v = *reinterpret_cast<const float4 *>(row + qd + kd + kc);
    const uint64_t idx = lbase + kv_index(page, 1, kc / hd, slot % 16, kc % hd, kv.n_kv, hd);
    put2(idx, v.x, v.y);
    put2(idx + 2, v.z, v.w);
  }
}

__global__ void k_rope_kv_batch(const float *qkv, uint32_t Hq, uint32_t Hkv, uint32_t hd, const float *rope,
                                uint32_t rope_max, const SeqState *st, KvView kv, uint32_t seq0, uint32_t layer,
                                float *qf, uint32_t *err) {
  pdl_enter();
  const uint32_t r = blockIdx.x, half = hd / 2, qd = Hq * hd, kd = Hkv * hd;
  const float *row = qkv + (size_t)r * (qd + 2 * kd);
  const uint32_t pos = st[r].pos, slot = st[r].len;
  if (pos >= rope_max || slot / 16 >= kv.max_pages) {
    if (threadIdx.x == 0 && err) atomicOr(err, kErrContext);
    return;
  }
  const float *cs = rope + (size_t)pos * hd;
  const uint32_t page = kv.page_table[(seq0 + r) * kv.max_pages + slot / 16];
  const uint64_t lbase = (uint64_t)layer * kv.layer_stride;
  const uint32_t n = qd + 2 * kd;
  constexpr uint32_t kU = 8;  // elements per thread per round, their loads issued together
  for (uint32_t j0 = threadIdx.x; j0 < n; j0 += kU * blockDim.x) {
    float v[kU], pv[kU], cth[kU], sth[kU];
#pragma unroll
    for (uint32_t u = 0; u < kU; ++u) {
      const uint32_t j = j0 + u * blockDim.x;
      v[u] = pv[u] = cth[u] = sth[u] = 0.0f;
      if (j < n) {
        v[u] = row[j];
        if (j < qd + kd) {  // q and k are rotated
          const uint32_t base = j < qd ? 0 : qd, dd = (j - base) % hd, hb = j - dd;
          cth[u] = cs[2 * (dd % half)];
          sth[u] = cs[2 * (dd % half) + 1];
          pv[u] = dd < half ? row[hb + dd + half] : row[hb + dd - half];
        }
      }
    }
#pragma unroll
    for (uint32_t u = 0; u < kU; ++u) {
      const uint32_t j = j0 + u * blockDim.x;
      if (j >= n) break;
      float x = v[u];
      const bool is_q = j < qd, is_k = !is_q && j < qd + kd;
      if (is_q || is_k) {
        const uint32_t dd = (j - (is_q ? 0 : qd)) % hd;
        x = dd < half ? __fsub_rn(__fmul_rn(x, cth[u]), __fmul_rn(pv[u], sth[u]))
                      : __fadd_rn(__fmul_rn(pv[u], sth[u]), __fmul_rn(x, cth[u]));
      }
      if (is_q) {
        qf[(size_t)r * qd + j] = x;
      } else {
        const uint32_t kc = is_k ? j - qd : j - qd - kd;
        const uint64_t idx = lbase + kv_index(page, is_k ? 0 : 1, kc / hd, slot % 16, kc % hd, kv.n_kv, hd);
        if (kv.f16) reinterpret_cast<__half *>(kv.base)[idx] = __float2half_rn(x);
        else reinterpret_cast<float *>(kv.base)[idx] = x;
      }
    }
  }
}

// after the sampler: positions advance, the sampled ids (already the next
// step's input tokens) go to the history
__global__ void k_batch_step_end(SeqState *st, uint32_t b, const uint32_t *ids, uint32_t *hist, uint32_t max_steps,
                                 uint32_t *step) {
  pdl_enter();
  const uint32_t s = *step;
  for (uint32_t r = threadIdx.x; r < b; r += blockDim.x) {
    st[r].pos += 1;
    st[r].len += 1;
    if (s < max_steps) hist[(size_t)s * b + r] = ids[r];
  }
  __syncthreads();
  if (threadIdx.x == 0) *step = s + 1;
}

template <uint32_t HD, bool F16>
int launch_attn_hd(const AttnRowsParams &p, cudaStream_t st) {
  const uint32_t smem = 2 * kAK * HD * 2;  // K and V tiles: 32 KB at head_dim 128
  const dim3 grid((p.T + kAQ - 1) / kAQ, p.Hq);
  return launch_pdl(k_attn_causal<HD, F16>, grid, dim3(128), smem, st, (const __half *)p.qh, p.T, p.Hq, p.Hkv,
                    p.len0, p.kv, p.seq, p.layer, p.scale_log2, (__half *)p.out);
}

}  // namespace

namespace {
template <uint32_t HD, bool F16, uint32_t REP>
void *decode_rows_fn() {
  return (void *)k_attn_decode_rows<HD, F16, REP>;
}
template <uint32_t HD, bool F16>
void *decode_rows_rep(uint32_t rep) {
  switch (rep) {
    case 1: return decode_rows_fn<HD, F16, 1>();
    case 2: return decode_rows_fn<HD, F16, 2>();
    case 4: return decode_rows_fn<HD, F16, 4>();
    case 8: return decode_rows_fn<HD, F16, 8>();
    default: return nullptr;
  }
}
void *pick_decode_rows(uint32_t hd, bool f16, uint32_t rep) {
  if (hd == 128) return f16 ? decode_rows_rep<128, true>(rep) : decode_rows_rep<128, false>(rep);
  if (hd == 64) return f16 ? decode_rows_rep<64, true>(rep) : decode_rows_rep<64, false>(rep);
  return nullptr;
}
}  // namespace

int attn_rows_init() {
  for (uint32_t hd : {64u, 128u})
    for (bool f16 : {false, true})
      for (uint32_t rep : {1u, 2u, 4u, 8u})
        if (cudaFuncSetAttribute(pick_decode_rows(hd, f16, rep), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(4 * 2 * kDT * hd * 2)))
          return -1;
  return 0;
}

int launch_attn_decode_rows(const AttnParams &p, cudaStream_t st) {
  const uint32_t hd = p.kv.head_dim, rep = p.n_heads / p.kv.n_kv;
  if (!p.row_states || p.n_heads % p.kv.n_kv || !p.splits) return -1;
  void *fn = pick_decode_rows(hd, p.kv.f16 != 0, rep);
  if (!fn) return -1;
  const float scale_log2 = p.scale * 1.4426950408889634f;
  void *args[] = {(void *)&p, (void *)&scale_log2};
  const dim3 grid(p.splits, p.kv.n_kv, p.q_rows);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = (size_t)4 * 2 * kDT * hd * 2;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args) == cudaSuccess ? 0 : -1;
}

int launch_embed_rows(const void *emb, int type, const uint32_t *tok, uint32_t T, uint32_t d, uint32_t vocab, float *x,
                      uint32_t *err, cudaStream_t st) {
  return launch_pdl(k_embed_rows, dim3(T), dim3(256), 0, st, (const uint8_t *)emb, type, tok, T, d, vocab, x, err);
}
int launch_norm_rows_h(const float *x, const float *w, float eps, uint32_t T, uint32_t d, void *out, uint32_t *err,
                       cudaStream_t st) {
  return launch_pdl(k_norm_rows_h, dim3(T), dim3(256), 0, st, x, w, eps, d, (__half *)out, err);
}
int launch_rope_kv_rows(const float *qkv, uint32_t T, uint32_t Hq, uint32_t Hkv, uint32_t hd, const float *rope,
                        uint32_t rope_max, uint32_t pos0, uint32_t len0, const KvView &kv, uint32_t seq, uint32_t layer,
                        void *qh, uint32_t *err, cudaStream_t st) {
  const auto a16 = [](const void *q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  if (hd % 4 == 0 && a16(qkv) && a16(rope) && a16(kv.base) && kv.layer_stride % 4 == 0 && reinterpret_cast<uintptr_t>(qh) % 4 == 0)
    return launch_pdl(k_rope_kv_rows4, dim3(T), dim3(256), 0, st, qkv, T, Hq, Hkv, hd, rope, rope_max, pos0, len0, kv,
                      seq, layer, (__half *)qh, err);
  return launch_pdl(k_rope_kv_rows, dim3(T), dim3(256), 0, st, qkv, T, Hq, Hkv, hd, rope, rope_max, pos0, len0, kv, seq,
                    layer, (__half *)qh, err);
}
int launch_attn_rows(const AttnRowsParams &p, cudaStream_t st) {
  if (p.Hq % p.Hkv) return -1;
  if (p.hd == 128) return p.kv.f16 ? launch_attn_hd<128, true>(p, st) : launch_attn_hd<128, false>(p, st);
  if (p.hd == 64) return p.kv.f16 ? launch_attn_hd<64, true>(p, st) : launch_attn_hd<64, false>(p, st);
  return -1;
}
int launch_swiglu_rows(const float *gu, uint32_t T, uint32_t F, uint32_t CW, void *h, uint32_t *err, cudaStream_t st) {
  if (F % 4 == 0 && CW % 32 == 0 && reinterpret_cast<uintptr_t>(gu) % 16 == 0 && reinterpret_cast<uintptr_t>(h) % 8 == 0)
    return launch_pdl(k_swiglu_rows4, dim3((F / 4 + 255) / 256, T), dim3(256), 0, st, gu, F, CW, (__half *)h, err);
  return launch_pdl(k_swiglu_rows, dim3((F + 255) / 256, T), dim3(256), 0, st, gu, F, CW, (__half *)h, err);
}
int launch_rope_kv_batch(const float *qkv, uint32_t b, uint32_t Hq, uint32_t Hkv, uint32_t hd, const float *rope,
                         uint32_t rope_max, const SeqState *states, const KvView &kv, uint32_t seq0, uint32_t layer,
                         float *qf, uint32_t *err, cudaStream_t st) {
  const auto a16 = [](const void *q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  if (hd % 4 == 0 && a16(qkv) && a16(rope) && a16(kv.base) && kv.layer_stride % 4 == 0 && reinterpret_cast<uintptr_t>(qf) % 8 == 0) {
    const uint32_t units = (Hq + Hkv) * (hd / 4) + Hkv * hd / 4;
    return launch_pdl(k_rope_kv_batch4, dim3(b, (units + 255) / 256), dim3(256), 0, st, qkv, Hq, Hkv, hd, rope, rope_max,
                      states, kv, seq0, layer, qf, err);
  }
  return launch_pdl(k_rope_kv_batch, dim3(b), dim3(256), 0, st, qkv, Hq, Hkv, hd, rope, rope_max, states, kv, seq0, layer,
                    qf, err);
}
int launch_batch_step_end(SeqState *states, uint32_t b, const uint32_t *ids, uint32_t *hist, uint32_t max_steps,
                          uint32_t *step, cudaStream_t st) {
  return launch_pdl(k_batch_step_end, dim3(1), dim3(256), 0, st, states, b, ids, hist, max_steps, step);
}
int launch_last_row(const float *X, uint32_t row, uint32_t d, float *x, float *ssq, uint32_t n_ssq, cudaStream_t st) {
  return launch_pdl(k_last_row, dim3(1), dim3(256), 0, st, X, row, d, x, ssq, n_ssq);
}

}  // namespace fa
