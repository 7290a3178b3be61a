// nccl_merge.cu -- sequence-split merge over NVLink: every rank holds a
// contiguous slice of each sequence's KV, computes the partial triple
// (m, l, o) of its slice (zl_paged_decode_partial), and the triples are
// all-gathered with NCCL into local HBM and merged by one kernel (the merge
// is not a sum, so it cannot ride an NCCL reduction).
//
// NCCL is opened at run time with dlopen("libnccl.so.2"): in a process that
// already loaded NCCL (e.g. through torch) the same library instance is used,
// and the shared library itself has no link-time NCCL dependency.
//
// Failure handling. The communicator is created non-blocking, and the gather
// buffer is sized once at zl_nccl_init, so a step allocates nothing and never
// synchronises the device. zl_nccl_merge records an event after its
// all-gathers; zl_nccl_wait (and zl_check_status, which calls it first) polls
// that event and ncclCommGetAsyncError against a deadline. A collective whose
// peer is gone never completes: at the deadline the communicator is aborted
// (ncclCommAbort stops its kernels), the call returns ZL_ERR_TIMEOUT, and
// every later zl_nccl_merge on the context returns ZL_ERR_NCCL. The context
// itself stays usable for single-GPU work.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "zl_internal.h"

namespace {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
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
    a.CommInitRankConfig = (decltype(a.CommInitRankConfig))dlsym(h, "ncclCommInitRankConfig");
    a.AllGather = (decltype(a.AllGather))dlsym(h, "ncclAllGather");
    a.GroupStart = (decltype(a.GroupStart))dlsym(h, "ncclGroupStart");
    a.GroupEnd = (decltype(a.GroupEnd))dlsym(h, "ncclGroupEnd");
    a.CommDestroy = (decltype(a.CommDestroy))dlsym(h, "ncclCommDestroy");
    a.CommAbort = (decltype(a.CommAbort))dlsym(h, "ncclCommAbort");
    a.CommGetAsyncError = (decltype(a.CommGetAsyncError))dlsym(h, "ncclCommGetAsyncError");
    a.GetErrorString = (decltype(a.GetErrorString))dlsym(h, "ncclGetErrorString");
    a.ok = a.GetUniqueId && a.CommInitRankConfig && a.AllGather && a.GroupStart && a.GroupEnd &&
           a.CommDestroy && a.CommAbort && a.CommGetAsyncError && a.GetErrorString;
  });
  return a;
}

using Clock = std::chrono::steady_clock;

// Non-blocking NCCL calls may return ncclInProgress: poll the communicator's
// state until it settles or the deadline passes.
ncclResult_t settle(ncclComm_t comm, ncclResult_t r, Clock::time_point deadline) {
  NcclApi& a = api();
  while (r == ncclInProgress) {
    if (Clock::now() > deadline) return ncclInProgress;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
    if (a.CommGetAsyncError(comm, &r) != ncclSuccess) return ncclInternalError;
  }
  return r;
}

void abort_comm(zl_ctx* ctx) {
  if (!ctx->nccl_comm) return;
  api().CommAbort(reinterpret_cast<ncclComm_t>(ctx->nccl_comm));
  ctx->nccl_comm = nullptr;
  ctx->nccl_pending = false;
  ctx->nccl_aborted = true;
}

}  // namespace

using namespace zl;

namespace zl {

zl_status nccl_wait_pending(zl_ctx* ctx, int timeout_ms) {
  if (!ctx->nccl_pending || !ctx->nccl_comm) return ZL_OK;
  NcclApi& a = api();
  ncclComm_t comm = reinterpret_cast<ncclComm_t>(ctx->nccl_comm);
  const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
  for (;;) {
    const cudaError_t q = cudaEventQuery(ctx->nccl_done);
    if (q == cudaSuccess) {
      ctx->nccl_pending = false;
      return ZL_OK;
    }
    if (q != cudaErrorNotReady)
      return set_error(ZL_ERR_CUDA, "nccl wait: %s", cudaGetErrorString(q));
    ncclResult_t ar = ncclSuccess;
    if (a.CommGetAsyncError(comm, &ar) != ncclSuccess || (ar != ncclSuccess && ar != ncclInProgress)) {
      const char* why = a.GetErrorString(ar);
      abort_comm(ctx);
      return set_error(ZL_ERR_NCCL, "NCCL reported an asynchronous error (%s); communicator aborted", why);
    }
    if (Clock::now() > deadline) {
      abort_comm(ctx);
      return set_error(ZL_ERR_TIMEOUT,
                       "the sequence-split all-gather did not finish within %d ms (a peer rank is gone "
                       "or stalled); communicator aborted", timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

}  // namespace zl

#define ZL_NCCL_TRY(comm, expr, deadline)                                                  \
  do {                                                                                     \
    ncclResult_t _r = settle((comm), (expr), (deadline));                                  \
    if (_r != ncclSuccess)                                                                 \
      return set_error(ZL_ERR_NCCL, "%s failed: %s", #expr,                                \
                       _r == ncclInProgress ? "still in progress at the deadline"          \
                                            : api().GetErrorString(_r));                   \
  } while (0)

extern "C" {

zl_status zl_nccl_get_unique_id(uint8_t id_out[128]) {
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  NcclApi& a = api();
  if (!a.ok) return set_error(ZL_ERR_NCCL, "libnccl.so.2 could not be loaded: %s", dlerror());
  if (!id_out) return set_error(ZL_ERR_INVALID_ARG, "id_out is null");
  ncclUniqueId id;
  ncclResult_t r = a.GetUniqueId(&id);
  if (r != ncclSuccess) return set_error(ZL_ERR_NCCL, "ncclGetUniqueId: %s", a.GetErrorString(r));
  memcpy(id_out, &id, sizeof(id));
  return ZL_OK;
}

zl_status zl_nccl_init(zl_ctx* ctx, const uint8_t id[128], int nranks, int rank, int64_t max_rows,
                       int max_head_dim, int timeout_ms) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  NcclApi& a = api();
  if (!a.ok) return set_error(ZL_ERR_NCCL, "libnccl.so.2 could not be loaded");
  if (!id || nranks <= 0 || rank < 0 || rank >= nranks || max_rows <= 0 || max_head_dim <= 0 ||
      timeout_ms <= 0)
    return set_error(ZL_ERR_INVALID_ARG, "nccl_init: bad arguments (rank %d of %d, %lld rows, d %d, %d ms)",
                     rank, nranks, (long long)max_rows, max_head_dim, timeout_ms);
  if (ctx->nccl_comm) return set_error(ZL_ERR_INVALID_ARG, "nccl_init: already initialised");
  // The whole gather buffer up front: a step never allocates or synchronises.
  const size_t bytes = (size_t)nranks * (size_t)max_rows * (2 + (size_t)max_head_dim) * sizeof(float);
  if (ctx->gather_buf) {
    cudaFree(ctx->gather_buf);
    ctx->gather_buf = nullptr;
    ctx->gather_bytes = 0;
  }
  ZL_CUDA_TRY(cudaMalloc(&ctx->gather_buf, bytes));
  ctx->gather_bytes = bytes;
  if (!ctx->nccl_done) ZL_CUDA_TRY(cudaEventCreateWithFlags(&ctx->nccl_done, cudaEventDisableTiming));
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  // Creating the communicator waits for every rank: allow it ten timeouts.
  const auto deadline = Clock::now() + std::chrono::milliseconds(10LL * timeout_ms);
  ncclResult_t r = a.CommInitRankConfig(&comm, nranks, uid, rank, &cfg);
  if (r == ncclInProgress) r = settle(comm, r, deadline);
  if (r != ncclSuccess) {
    if (comm) a.CommAbort(comm);
    return set_error(r == ncclInProgress ? ZL_ERR_TIMEOUT : ZL_ERR_NCCL,
                     "ncclCommInitRankConfig (rank %d of %d): %s", rank, nranks,
                     r == ncclInProgress ? "not every rank joined in time" : a.GetErrorString(r));
  }
  ctx->nccl_comm = comm;
  ctx->nranks = nranks;
  ctx->rank = rank;
  ctx->nccl_max_rows = max_rows;
  ctx->nccl_max_d = max_head_dim;
  ctx->nccl_timeout_ms = timeout_ms;
  ctx->nccl_pending = false;
  ctx->nccl_aborted = false;
  return ZL_OK;
}

zl_status zl_nccl_merge(zl_ctx* ctx, const float* m, const float* l, const float* o, int64_t rows,
                        int head_dim, void* out, zl_dtype dtype, zl_stream stream) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  if (ctx->nccl_aborted)
    return set_error(ZL_ERR_NCCL, "nccl_merge: the communicator was aborted after a lost peer");
  if (!ctx->nccl_comm) return set_error(ZL_ERR_NCCL, "nccl_merge: call zl_nccl_init first");
  if (rows < 0 || head_dim <= 0 || !dtype_ok(dtype))
    return set_error(ZL_ERR_INVALID_ARG, "nccl_merge: bad arguments");
  if (rows > ctx->nccl_max_rows || head_dim > ctx->nccl_max_d)
    return set_error(ZL_ERR_INVALID_ARG,
                     "nccl_merge: %lld rows x d %d exceed the gather buffer sized at zl_nccl_init "
                     "(%lld rows x d %d)", (long long)rows, head_dim, (long long)ctx->nccl_max_rows,
                     ctx->nccl_max_d);
  if (rows == 0) return ZL_OK;
  if (!m || !l || !o || !out) return set_error(ZL_ERR_INVALID_ARG, "nccl_merge: null pointer");
  const int P = ctx->nranks;
  float* gm = reinterpret_cast<float*>(ctx->gather_buf);   // [P][rows]
  float* gl = gm + (size_t)P * rows;                        // [P][rows]
  float* go = gl + (size_t)P * rows;                        // [P][rows][d]
  NcclApi& a = api();
  cudaStream_t st = S(stream);
  ncclComm_t comm = reinterpret_cast<ncclComm_t>(ctx->nccl_comm);
  const auto deadline = Clock::now() + std::chrono::milliseconds(ctx->nccl_timeout_ms);
  ZL_NCCL_TRY(comm, a.GroupStart(), deadline);
  ZL_NCCL_TRY(comm, a.AllGather(m, gm, (size_t)rows, ncclFloat32, comm, st), deadline);
  ZL_NCCL_TRY(comm, a.AllGather(l, gl, (size_t)rows, ncclFloat32, comm, st), deadline);
  ZL_NCCL_TRY(comm, a.AllGather(o, go, (size_t)rows * head_dim, ncclFloat32, comm, st), deadline);
  ZL_NCCL_TRY(comm, a.GroupEnd(), deadline);
  ZL_CUDA_TRY(cudaEventRecord(ctx->nccl_done, st));
  ctx->nccl_pending = true;
  return launch_merge(ctx, gm, gl, go, P, rows, head_dim, out, dtype, st);
}

zl_status zl_nccl_wait(zl_ctx* ctx, int timeout_ms) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  if (ctx->nccl_aborted)
    return set_error(ZL_ERR_NCCL, "nccl_wait: the communicator was aborted after a lost peer");
  return nccl_wait_pending(ctx, timeout_ms > 0 ? timeout_ms : ctx->nccl_timeout_ms);
}

zl_status zl_nccl_abort(zl_ctx* ctx) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  abort_comm(ctx);
  return ZL_OK;
}

zl_status zl_nccl_finalize(zl_ctx* ctx) {
  if (!ctx) return ZL_OK;
  cudaSetDevice(ctx->device);
  if (ctx->nccl_comm) {
    // A collective that cannot finish is aborted rather than waited for.
    if (nccl_wait_pending(ctx, ctx->nccl_timeout_ms) == ZL_OK && ctx->nccl_comm) {
      NcclApi& a = api();
      ncclComm_t comm = reinterpret_cast<ncclComm_t>(ctx->nccl_comm);
      const auto deadline = Clock::now() + std::chrono::milliseconds(ctx->nccl_timeout_ms);
      if (settle(comm, a.CommDestroy(comm), deadline) != ncclSuccess) a.CommAbort(comm);
    }
  }
  ctx->nccl_comm = nullptr;
  ctx->nccl_pending = false;
  ctx->nccl_aborted = false;
  ctx->nranks = 1;
  ctx->rank = 0;
  if (ctx->gather_buf) {
    cudaFree(ctx->gather_buf);
    ctx->gather_buf = nullptr;
    ctx->gather_bytes = 0;
  }
  if (ctx->nccl_done) {
    cudaEventDestroy(ctx->nccl_done);
    ctx->nccl_done = nullptr;
  }
  return ZL_OK;
}

}  // extern "C"
