// Tensor-parallel shards and the NCCL communicator (see tp.hpp).
#include "tp.hpp"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "fa_host.hpp"
#include "fa_layout.hpp"

namespace fa {

// ---------------------------------------------------------------------------
// shards
// ---------------------------------------------------------------------------
namespace {

// the 6-bit (scale, min) pair of Q4_K sub-block j from the 12 packed bytes
void q4k_pair(const uint8_t *q, int j, int *sc, int *m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// half h (columns [128h, 128h + 128)) of a 144-byte Q4_K block -> a block
// whose columns [0, 128) dequantise to the same values and [128, 256) to 0
void q4k_half_block(const uint8_t *b, int h, uint8_t *o) {
  std::memcpy(o, b, 4);  // d, dmin
  uint8_t *sc = o + 4;
  std::memset(sc, 0, 12);
  for (int j = 0; j < 4; ++j) {
    int s, m;
    q4k_pair(b + 4, 4 * h + j, &s, &m);
    sc[j] = (uint8_t)s;  // sub-blocks 4-7 are zero, so no high bits to spread
    sc[j + 4] = (uint8_t)m;
  }
  std::memcpy(o + 16, b + 16 + 64 * h, 64);  // codes of 64-column pieces 2h, 2h+1
  std::memset(o + 80, 0, 64);
}

}  // namespace

int tp_shard_columns(int type, const uint8_t *src, uint32_t K, uint32_t N, uint32_t c0, uint32_t c1,
                     std::vector<uint8_t> &out, uint32_t *row_bytes) {
  if (c0 >= c1 || c1 > N || !type_known(type)) return -1;
  const uint32_t bs = (uint32_t)block_elems(type), bb = (uint32_t)block_bytes(type);
  const uint64_t src_rb = (uint64_t)N / bs * bb;
  if (c0 % bs == 0 && c1 % bs == 0) {
    const uint32_t rb = (c1 - c0) / bs * bb;
    out.resize((uint64_t)K * rb);
    for (uint32_t k = 0; k < K; ++k) std::memcpy(out.data() + (uint64_t)k * rb, src + k * src_rb + c0 / bs * bb, rb);
    *row_bytes = rb;
    return 0;
  }
  if (type == kQ4_K && c1 - c0 == 128 && c0 % 128 == 0) {
    out.resize((uint64_t)K * 144);
    for (uint32_t k = 0; k < K; ++k)
      q4k_half_block(src + k * src_rb + (c0 / 256) * 144, (c0 % 256) / 128, out.data() + (uint64_t)k * 144);
    *row_bytes = 144;
    return 0;
  }
  return -1;
}

// ---------------------------------------------------------------------------
// NCCL, loaded on first use
// ---------------------------------------------------------------------------
namespace {

struct NcclApi {
  bool tried = false, ok = false;
  std::string err;
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

std::mutex g_nccl_mu;
NcclApi g_nccl;

const NcclApi *nccl(std::string *msg) {
  std::lock_guard<std::mutex> lock(g_nccl_mu);
  NcclApi &a = g_nccl;
  if (!a.tried) {
    a.tried = true;
    // a process that already loaded NCCL (e.g. through its framework) gets
    // that copy back from the loader
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      a.err = std::string("libnccl.so.2 not found: ") + dlerror();
    } else {
      a.GetUniqueId = (decltype(a.GetUniqueId))dlsym(h, "ncclGetUniqueId");
      a.CommInitRank = (decltype(a.CommInitRank))dlsym(h, "ncclCommInitRank");
      a.AllReduce = (decltype(a.AllReduce))dlsym(h, "ncclAllReduce");
      a.CommDestroy = (decltype(a.CommDestroy))dlsym(h, "ncclCommDestroy");
      a.CommAbort = (decltype(a.CommAbort))dlsym(h, "ncclCommAbort");
      a.CommGetAsyncError = (decltype(a.CommGetAsyncError))dlsym(h, "ncclCommGetAsyncError");
      a.GetErrorString = (decltype(a.GetErrorString))dlsym(h, "ncclGetErrorString");
      a.ok = a.GetUniqueId && a.CommInitRank && a.AllReduce && a.CommDestroy && a.CommAbort && a.CommGetAsyncError &&
             a.GetErrorString;
      if (!a.ok) a.err = "libnccl.so.2 lacks an expected entry point";
    }
  }
  if (!a.ok) {
    if (msg) *msg = a.err;
    return nullptr;
  }
  return &a;
}

std::string nccl_msg(const NcclApi *a, ncclResult_t r) { return a->GetErrorString ? a->GetErrorString(r) : "nccl error"; }

}  // namespace

int tp_unique_id(void *out128, std::string *msg) {
  const NcclApi *a = nccl(msg);
  if (!a) return -1;
  ncclUniqueId id;
  const ncclResult_t r = a->GetUniqueId(&id);
  if (r != ncclSuccess) {
    if (msg) *msg = nccl_msg(a, r);
    return -1;
  }
  std::memcpy(out128, id.internal, NCCL_UNIQUE_ID_BYTES);
  return 0;
}

TpComm::~TpComm() {
  if (!comm) return;
  if (const NcclApi *a = nccl(nullptr)) a->CommDestroy((ncclComm_t)comm);
  comm = nullptr;
}

int TpComm::init(int r, int w, const void *uid, int device) {
  std::string msg;
  const NcclApi *a = nccl(&msg);
  if (!a) return fail(FA_ERR_NCCL, msg);
  if (cudaSetDevice(device) != cudaSuccess) return fail(FA_ERR_CUDA, "cudaSetDevice failed");
  ncclUniqueId id;
  std::memcpy(id.internal, uid, NCCL_UNIQUE_ID_BYTES);
  ncclComm_t c = nullptr;
  const ncclResult_t res = a->CommInitRank(&c, w, id, r);
  if (res != ncclSuccess) return fail(FA_ERR_NCCL, "ncclCommInitRank: " + nccl_msg(a, res));
  comm = c;
  rank = r;
  world = w;
  return FA_OK;
}

int TpComm::all_reduce(const float *send, float *recv, size_t count, cudaStream_t st) {
  const NcclApi *a = nccl(nullptr);
  if (!a || !comm) return fail(FA_ERR_NCCL, "no NCCL communicator");
  const ncclResult_t r = a->AllReduce(send, recv, count, ncclFloat32, ncclSum, (ncclComm_t)comm, st);
  return r == ncclSuccess ? FA_OK : fail(FA_ERR_NCCL, "ncclAllReduce: " + nccl_msg(a, r));
}

int TpComm::check_async(std::string *msg) {
  const NcclApi *a = nccl(nullptr);
  if (!a || !comm) return 0;
  ncclResult_t r = ncclSuccess;
  if (a->CommGetAsyncError((ncclComm_t)comm, &r) != ncclSuccess) r = ncclSystemError;
  if (r == ncclSuccess || r == ncclInProgress) return 0;
  if (msg) *msg = nccl_msg(a, r);
  abort();
  return -1;
}

void TpComm::abort() {
  if (!comm) return;
  if (const NcclApi *a = nccl(nullptr)) a->CommAbort((ncclComm_t)comm);
  comm = nullptr;
}

}  // namespace fa
