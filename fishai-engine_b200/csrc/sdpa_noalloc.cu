// fa_sdpa_noalloc: the split-K attention of fa_sdpa for callers that must
// not allocate device memory — for example code running where a cudaMalloc
// would break the surrounding contract: a host thread that only holds
// pre-reserved memory under an external allocator's budget, or a latency
// path where a synchronous allocation (which can stall the whole device) is
// not acceptable.  Its scratch (split partials + arrival counters) lives in
// a file-scope __device__ array of fixed size that every GPU loading this
// library holds until the process exits; nothing here calls cudaMalloc,
// cudaFree or an allocating library routine.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/fishai_cuda.h"
#include "fa_host.hpp"
#include "fa_kernels.hpp"
#include "sdpa.hpp"

namespace {

constexpr size_t kMaxPartFloats = 1u << 19;    // 2 MiB of split partials
constexpr size_t kMaxCounters = 1024;          // q_len * n_kv_heads arrival counters
constexpr size_t kScratchFloats = kMaxPartFloats + kMaxCounters;

// the only scratch the entry point uses; shared by every call on a device
static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

std::mutex g_mu;
float *g_addr[64];  // device address of g_noalloc_scratch per device ordinal

}  // namespace

extern "C" int fa_sdpa_noalloc(const float *q, const float *k, const float *v, uint32_t q_len, uint32_t kv_len,
                               uint32_t H, uint32_t KVH, uint32_t hd, float *out, void *stream) {
  using namespace fa;
  int rc = sdpa_check("fa_sdpa_noalloc", q, k, v, q_len, kv_len, H, KVH, hd, out);
  if (rc) return rc;
  // the limits follow fa_sdpa's split count (kSdpaSplits)
  const uint64_t part_floats = sdpa_part_floats(q_len, H, hd);
  const uint64_t counters = sdpa_counters(q_len, KVH);
  if (part_floats > kMaxPartFloats || counters > kMaxCounters)
    return fail(FA_ERR_INVALID, "fa_sdpa_noalloc: q_len*n_heads*" + std::to_string(kSdpaSplits) +
                                    "*(head_dim+2) = " + std::to_string(part_floats) +
                                    " exceeds the fixed scratch of " + std::to_string(kMaxPartFloats) +
                                    " floats, or q_len*n_kv_heads = " + std::to_string(counters) + " exceeds " +
                                    std::to_string(kMaxCounters));
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(FA_ERR_CUDA, "fa_sdpa_noalloc: no current CUDA device");
  float *base;
  {
    // first call on a device: resolve the array's device address with that
    // device current (a host-side name of a __device__ variable is not a
    // device pointer)
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[dev]) {
      void *p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p)
        return fail(FA_ERR_CUDA, std::string("fa_sdpa_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
      g_addr[dev] = (float *)p;
    }
    base = g_addr[dev];
  }
  float *part = base;
  uint32_t *cnt = reinterpret_cast<uint32_t *>(base + kMaxPartFloats);
  // the arrival counters must start at zero; the array keeps the last call's contents
  if (cudaMemsetAsync(cnt, 0, counters * sizeof(uint32_t), (cudaStream_t)stream) != cudaSuccess)
    return fail(FA_ERR_CUDA, "fa_sdpa_noalloc: clearing the counters failed");
  const AttnParams ap = sdpa_params(q, k, v, q_len, kv_len, H, KVH, hd, out, part, cnt);
  if (launch_attention(ap, false, (cudaStream_t)stream)) return fail(FA_ERR_CUDA, "fa_sdpa_noalloc: launch failed");
  return FA_OK;
}
