// Tensor-core dequant-GEMV for batch-1 decode, y[N] = x[K] . W[K][N] for
// Q4_K, Q6_K, Q8_0 and Q4_0 weights in the MMA tile layout (fa_layout.hpp),
// the reference's tensor::matmul orientation (src/tensor.rs:244-258).
//
// The multiply-add of every weight element runs on the tensor pipe as
// mma.sync.m16n8k16 (bf16 in, f32 accumulate) with the weight codes as
// operand A and per-row coefficients as operand B:
//   * A: a weight code q (4, 6 or 8 bits) masked into the low bits of a bf16
//     half is the bf16 subnormal q * 2^-133 — exact, one LOP3 per two codes,
//     no conversion and no bias to subtract;
//   * B: c = x[k] * d[k] * sc[k][block] (the dequantisation scale of row k
//     for the tile's block times the activation), times 2^96, split exactly
//     into three bf16 (hi + mid + lo = 24 bits) held in B columns 0..2.
// D[m][0] + D[m][1] + D[m][2] = 2^-37 * sum_k q[k][m] * c[k]; the constant
// parts of the dequantisation (Q4_K mins, the Q6_K/Q8_0/Q4_0 code offsets)
// are per-block sums of c (or x*dmin*m) kept in f32 beside the MMA.
//
// Work split: persistent CTAs (one per SM) stream byte-balanced ranges of
// (chunk, 16-row group) units (stream-K).  A producer lane fills a shared-
// memory ring (as many slots as fit, up to 12) with one large 1-D bulk copy
// per stage (up to four groups, ~32 KB: per-copy overhead makes small copies
// slow); weights are static, so it never waits for the previous kernel.  The
// consumers load the CTA's slice of x once (normalised when the launch has an
// RMSNorm prologue); each of the 16 consumer warps owns one 64-column slice
// of the 1024-wide chunk, builds the B coefficients of its slice for the stage
// in a private table and runs 4 (Q6_K: 8) MMAs per group.
// At the end of its rows of a chunk a CTA either adds its piece straight into
// the destination with one vector red.add per lane (kEpiRed, the decode
// step's form: the epilogue work moves into the next launch's prologue), or
// publishes the chunk partial and the last CTA to arrive sums the partials in
// a fixed order and runs the fused epilogue (gemv_epi.cuh).
#include "gemv_mma.cuh"

namespace fa {

using namespace mma;

__global__ void __launch_bounds__(kThreads, 1) k_gemv_mma(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Smem sm = carve(smem, p);
  const uint32_t tid = threadIdx.x, warp = tid / 32, lane = tid % 32;

  if (tid == 0) {
    for (uint32_t i = 0; i < p.n_stages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kWarps);
    }
    fence_mbar_init();
  }
  for (uint32_t i = tid; i < kZeroWords; i += kThreads) sm.zero[i] = 0u;
  __syncthreads();
  pdl_launch_dependents();

  bool ok = true;
  if (warp == kWarps) {
    // producer: weights only (static, so no wait on the previous kernel)
    uint32_t s = 0;
    if (lane == 0) produce(p, blockIdx.x, sm, s, ok);
  } else {
    pdl_wait();
    uint32_t slot = 0, phase = 0;
    consume(p, blockIdx.x, sm, tid, warp, lane, slot, phase, ok);
  }
  if (!ok && p.state) atomicOr(&p.state->err, kErrWaitTimeout);
}

uint32_t gemv_mma_stage_groups(uint32_t gbytes, int type) { return stage_groups(gbytes, type); }
uint32_t gemv_mma_table_offset() { return kOffTbl; }
uint32_t gemv_mma_table_words() { return kWarps * kTblWords; }
uint32_t gemv_mma_ring_offset(uint32_t max_units) { return ring_offset(max_units); }

size_t gemv_mma_smem_bytes(const GemvParams &p) {
  return ring_offset(p.max_units) + (size_t)p.n_stages * p.stage_bytes;
}

uint32_t gemv_mma_stages(uint32_t stage_bytes, uint32_t max_units, size_t smem_budget) {
  const size_t fixed = ring_offset(max_units);
  const size_t n = smem_budget > fixed ? (smem_budget - fixed) / stage_bytes : 0;
  return (uint32_t)(n > kMaxStages ? kMaxStages : n);
}

int gemv_mma_init() {
  if (cudaFuncSetAttribute(k_gemv_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
    return -1;
  return 0;
}

int launch_gemv_mma(const GemvParams &p, bool pdl, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_ctas);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = gemv_mma_smem_bytes(p);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_gemv_mma, p) == cudaSuccess ? 0 : -1;
}

}  // namespace fa
