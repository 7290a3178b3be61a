// nccl_merge.cu -- sequence-split merge over NVLink: every rank holds a
// contiguous slice of each sequence's KV, computes the partial triple
// (m, l, o) of its slice (zl_paged_decode_partial), and the triples are
// all-gathered with NCCL into local HBM and merged by one kernel (the merge
// is not a sum, so it cannot ride an NCCL reduction).
//
// NCCL is opened at run time with dlopen("libnccl.so.2"): in a process that
// already loaded NCCL (e.g. through torch) the same library instance is used,
// and the shared library itself has no link-time NCCL dependency.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "zl_internal.h"

namespace {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

NcclApi& api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    a.handle = h;
    a.GetUniqueId = (decltype(a.GetUniqueId))dlsym(h, "ncclGetUniqueId");
    a.CommInitRank = (decltype(a.CommInitRank))dlsym(h, "ncclCommInitRank");
    a.AllGather = (decltype(a.AllGather))dlsym(h, "ncclAllGather");
    a.GroupStart = (decltype(a.GroupStart))dlsym(h, "ncclGroupStart");
    a.GroupEnd = (decltype(a.GroupEnd))dlsym(h, "ncclGroupEnd");
    a.CommDestroy = (decltype(a.CommDestroy))dlsym(h, "ncclCommDestroy");
    a.GetErrorString = (decltype(a.GetErrorString))dlsym(h, "ncclGetErrorString");
    a.ok = a.GetUniqueId && a.CommInitRank && a.AllGather && a.GroupStart && a.GroupEnd &&
           a.CommDestroy && a.GetErrorString;
  });
  return a;
}

}  // namespace

using namespace zl;

#define ZL_NCCL_TRY(expr)                                                                  \
  do {                                                                                     \
    ncclResult_t _r = (expr);                                                              \
    if (_r != ncclSuccess)                                                                 \
      return set_error(ZL_ERR_NCCL, "%s failed: %s", #expr, api().GetErrorString(_r));     \
  } while (0)

extern "C" {

zl_status zl_nccl_get_unique_id(uint8_t id_out[128]) {
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  NcclApi& a = api();
  if (!a.ok) return set_error(ZL_ERR_NCCL, "libnccl.so.2 could not be loaded: %s", dlerror());
  if (!id_out) return set_error(ZL_ERR_INVALID_ARG, "id_out is null");
  ncclUniqueId id;
  ZL_NCCL_TRY(a.GetUniqueId(&id));
  memcpy(id_out, &id, sizeof(id));
  return ZL_OK;
}

zl_status zl_nccl_init(zl_ctx* ctx, const uint8_t id[128], int nranks, int rank) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  NcclApi& a = api();
  if (!a.ok) return set_error(ZL_ERR_NCCL, "libnccl.so.2 could not be loaded");
  if (!id || nranks <= 0 || rank < 0 || rank >= nranks)
    return set_error(ZL_ERR_INVALID_ARG, "nccl_init: bad rank %d of %d", rank, nranks);
  if (ctx->nccl_comm) return set_error(ZL_ERR_INVALID_ARG, "nccl_init: already initialised");
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t comm = nullptr;
  ZL_NCCL_TRY(a.CommInitRank(&comm, nranks, uid, rank));
  ctx->nccl_comm = comm;
  ctx->nranks = nranks;
  ctx->rank = rank;
  return ZL_OK;
}

zl_status zl_nccl_merge(zl_ctx* ctx, const float* m, const float* l, const float* o, int64_t rows,
                        int head_dim, void* out, zl_dtype dtype, zl_stream stream) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  if (!ctx->nccl_comm) return set_error(ZL_ERR_NCCL, "nccl_merge: call zl_nccl_init first");
  if (rows < 0 || head_dim <= 0 || !dtype_ok(dtype))
    return set_error(ZL_ERR_INVALID_ARG, "nccl_merge: bad arguments");
  if (rows == 0) return ZL_OK;
  if (!m || !l || !o || !out) return set_error(ZL_ERR_INVALID_ARG, "nccl_merge: null pointer");
  const int P = ctx->nranks;
  const size_t per_rank = (size_t)rows * (2 + head_dim);
  const size_t bytes = per_rank * P * sizeof(float);
  if (bytes > ctx->gather_bytes) {
    if (ctx->gather_buf) {
      ZL_CUDA_TRY(cudaDeviceSynchronize());
      ZL_CUDA_TRY(cudaFree(ctx->gather_buf));
      ctx->gather_buf = nullptr;
    }
    ZL_CUDA_TRY(cudaMalloc(&ctx->gather_buf, bytes));
    ctx->gather_bytes = bytes;
  }
  float* gm = reinterpret_cast<float*>(ctx->gather_buf);   // [P][rows]
  float* gl = gm + (size_t)P * rows;                        // [P][rows]
  float* go = gl + (size_t)P * rows;                        // [P][rows][d]
  NcclApi& a = api();
  cudaStream_t st = S(stream);
  ncclComm_t comm = reinterpret_cast<ncclComm_t>(ctx->nccl_comm);
  ZL_NCCL_TRY(a.GroupStart());
  ZL_NCCL_TRY(a.AllGather(m, gm, (size_t)rows, ncclFloat32, comm, st));
  ZL_NCCL_TRY(a.AllGather(l, gl, (size_t)rows, ncclFloat32, comm, st));
  ZL_NCCL_TRY(a.AllGather(o, go, (size_t)rows * head_dim, ncclFloat32, comm, st));
  ZL_NCCL_TRY(a.GroupEnd());
  return launch_merge(ctx, gm, gl, go, P, rows, head_dim, out, dtype, st);
}

zl_status zl_nccl_finalize(zl_ctx* ctx) {
  if (!ctx || !ctx->nccl_comm) return ZL_OK;
  cudaSetDevice(ctx->device);
  cudaDeviceSynchronize();
  NcclApi& a = api();
  if (a.ok) a.CommDestroy(reinterpret_cast<ncclComm_t>(ctx->nccl_comm));
  ctx->nccl_comm = nullptr;
  ctx->nranks = 1;
  ctx->rank = 0;
  return ZL_OK;
}

}  // extern "C"
