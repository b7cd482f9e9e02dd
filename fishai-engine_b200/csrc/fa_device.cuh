// Device helpers for sm_100a: mbarriers with bounded waits, 1-D bulk TMA
// copies (cp.async.bulk, no multicast), cluster / DSMEM access,
// programmatic dependent launch, packed f32x2 FMA, f16 conversion.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "fa_kernels.hpp"

namespace fa {

// Spin budget for one mbarrier wait: try_wait suspends for a while on each
// call, so ~2^22 tries is well beyond any legitimate wait (seconds).
constexpr uint32_t kMaxWaitTries = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Arrival on a GPU-scope counter with acquire-release semantics: the caller's
// CTA writes ordered before it by a barrier are released with it, and the
// arriver that sees the final count acquires every other arriver's writes
// (a following barrier passes them on to the rest of its CTA).
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t *p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void red_add_release_gpu(uint32_t *p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait on phase `parity`.  Returns false (and the caller must set an
// error flag and unwind) if the barrier did not complete within the budget.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < kMaxWaitTries; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait on phase `parity` with the thread suspended between polls (the
// hardware wakes it when the phase completes, so polling is rare); gives up
// and returns false after `limit_ns` of wall time.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far beyond any legitimate wait
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs) {
  const uint32_t addr = smem_u32(bar);
  uint64_t t0 = 0;
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity), "r"(1000000u)
        : "memory");
    if (done) return true;
    const uint64_t t = global_ns();
    if (!t0) t0 = t;
    else if (t - t0 > limit_ns) return false;
  }
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes).
// src, dst 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch (no-ops when the launch has no PDL attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }
// first statement of a kernel launched by launch_pdl: let the next kernel's
// CTAs be scheduled, then wait for the previous kernels' completion (and
// their memory) before touching anything they write or read
__device__ __forceinline__ void pdl_enter() {
  pdl_launch_dependents();
  pdl_wait();
}

// Launch with programmatic dependent launch: the kernel's CTAs may start
// while the previous kernel on the stream finishes, so the kernel must call
// pdl_wait() (pdl_enter()) before it uses memory earlier kernels write or read.
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args &&>(args)...) == cudaSuccess ? 0 : -1;
}

// ---- clusters / DSMEM ----
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// address of the same shared variable in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t dsmem_addr(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ float dsmem_ld_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// ---- arithmetic ----
// acc{0,1} += a{0,1} * b{0,1}, one packed Blackwell FFMA2
__device__ __forceinline__ void ffma2(float &acc0, float &acc1, float a0, float a1, float b0, float b1) {
  uint64_t acc = ((uint64_t)__float_as_uint(acc1) << 32) | __float_as_uint(acc0);
  uint64_t av = ((uint64_t)__float_as_uint(a1) << 32) | __float_as_uint(a0);
  uint64_t bv = ((uint64_t)__float_as_uint(b1) << 32) | __float_as_uint(b0);
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(av), "l"(bv));
  acc0 = __uint_as_float((uint32_t)acc);
  acc1 = __uint_as_float((uint32_t)(acc >> 32));
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// integer in [0, 2^23) to float without the (slow) I2F path: exact
__device__ __forceinline__ float u2f_small(uint32_t v) {
  return __uint_as_float(0x4B000000u | v) - 8388608.0f;
}

// orderable 32-bit key of a float (larger float -> larger key)
__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(b);
}

}  // namespace fa
