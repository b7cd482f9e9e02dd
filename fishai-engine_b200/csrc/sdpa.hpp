// Setup shared by the two entry points of the contiguous-K/V attention,
// fa_sdpa (library-allocated scratch) and fa_sdpa_noalloc (fixed static
// scratch): one split count, one argument check, one parameter fill, so the
// two give the same numbers for the same arguments.
#pragma once
#include <stdint.h>

#include "fa_kernels.hpp"

namespace fa {

constexpr uint32_t kSdpaSplits = 32;  // position splits per (query row, kv head)

// floats of split partials and counters one call needs
inline uint64_t sdpa_part_floats(uint32_t q_len, uint32_t H, uint32_t hd) {
  return (uint64_t)q_len * H * kSdpaSplits * (2 + hd);
}
inline uint64_t sdpa_counters(uint32_t q_len, uint32_t KVH) { return (uint64_t)q_len * KVH; }

// argument check; `who` names the entry point in the error message
int sdpa_check(const char *who, const float *q, const float *k, const float *v, uint32_t q_len, uint32_t kv_len,
               uint32_t H, uint32_t KVH, uint32_t hd, const float *out);
AttnParams sdpa_params(const float *q, const float *k, const float *v, uint32_t q_len, uint32_t kv_len, uint32_t H,
                       uint32_t KVH, uint32_t hd, float *out, float *part, uint32_t *counters);

}  // namespace fa
