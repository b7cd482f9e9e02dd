// Tensor parallelism (Megatron column / row shards of the layer projections)
// for the decode path: host-side shard extraction from the native GGUF
// blocks, and the NCCL communicator the all-reduces after the o and down
// projections run on.  NCCL is loaded at run time (libnccl.so.2), so models
// without tensor parallelism never touch it.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace fa {

// rows [r0, r1) of W[K][N] stored in native blocks: one contiguous range
inline const uint8_t *tp_rows(const uint8_t *src, uint32_t row_bytes, uint32_t r0) {
  return src + (uint64_t)r0 * row_bytes;
}

// Columns [c0, c1) of every row of W[K][N] (native blocks along N) copied into
// `out` as a [K][c1 - c0] tensor; *row_bytes receives its row stride.  Both
// ends must be multiples of the type's block, except that a Q4_K range of
// exactly 128 columns starting at a multiple of 128 (half of a 256-column
// super-block: one 128-wide KV head at eight-way parallelism) is re-encoded
// as one block holding that half in its lower 128 columns (same d and dmin,
// the half's four 6-bit scale/min pairs moved to sub-blocks 0-3, its 64 code
// bytes first) and zeros above: the half dequantises to exactly the same
// values.  Returns 0, or -1 for a range the rules do not allow.
int tp_shard_columns(int type, const uint8_t *src, uint32_t K, uint32_t N, uint32_t c0, uint32_t c1,
                     std::vector<uint8_t> &out, uint32_t *row_bytes);

// NCCL communicator of one rank (dlopen'd libnccl.so.2).
struct TpComm {
  void *comm = nullptr;  // ncclComm_t
  int rank = 0, world = 1;
  ~TpComm();
  int init(int rank, int world, const void *unique_id_128, int device);
  // sum of `count` floats over the ranks, send -> recv (in place when equal)
  int all_reduce(const float *send, float *recv, size_t count, cudaStream_t st);
  // the communicator's asynchronous error (0 = none); aborts it on error
  int check_async(std::string *msg);
  void abort();
};

// 128-byte ncclUniqueId for rank 0 to share with the others
int tp_unique_id(void *out128, std::string *msg);

}  // namespace fa
