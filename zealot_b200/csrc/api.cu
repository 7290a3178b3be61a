// api.cu -- context lifetime, error reporting and the device status word.
//
// zl_ctx replaces GpuContext (src/gpu_context.rs:16-52 of the reference): it
// binds a device and owns the only library-side device memory (status word,
// split-KV workspace, self-resetting counters). Everything else belongs to
// the caller.
#include "zl_internal.h"

#include <cstdlib>
#include <cstring>

namespace zl {

static thread_local std::string g_last_error;

zl_status set_error(zl_status s, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

zl_status bind_device(zl_ctx* ctx) {
  if (!ctx) return set_error(ZL_ERR_INVALID_ARG, "null context");
  ZL_CUDA_TRY(cudaSetDevice(ctx->device));
  return ZL_OK;
}

zl_status ensure_workspace(zl_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->workspace_bytes) return ZL_OK;
  if (ctx->workspace) {
    // The old buffer may still be read by in-flight kernels on any stream.
    ZL_CUDA_TRY(cudaDeviceSynchronize());
    ZL_CUDA_TRY(cudaFree(ctx->workspace));
    ctx->workspace = nullptr;
    ctx->workspace_bytes = 0;
  }
  size_t sz = bytes + bytes / 4 + 4096;
  ZL_CUDA_TRY(cudaMalloc(&ctx->workspace, sz));
  ctx->workspace_bytes = sz;
  return ZL_OK;
}

zl_status ensure_counters(zl_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->counters_bytes) return ZL_OK;
  if (ctx->counters) {
    ZL_CUDA_TRY(cudaDeviceSynchronize());
    ZL_CUDA_TRY(cudaFree(ctx->counters));
    ctx->counters = nullptr;
    ctx->counters_bytes = 0;
  }
  size_t sz = bytes + bytes / 4 + 4096;
  ZL_CUDA_TRY(cudaMalloc(&ctx->counters, sz));
  // Counters start at zero and every kernel that uses one returns it to zero.
  ZL_CUDA_TRY(cudaMemset(ctx->counters, 0, sz));
  ZL_CUDA_TRY(cudaDeviceSynchronize());
  ctx->counters_bytes = sz;
  return ZL_OK;
}

}  // namespace zl

using namespace zl;

extern "C" {

int zl_abi_version(void) { return ZL_ABI_VERSION; }

const char* zl_last_error(void) { return g_last_error.c_str(); }

const char* zl_status_string(zl_status s) {
  switch (s) {
    case ZL_OK: return "ok";
    case ZL_ERR_INVALID_ARG: return "invalid argument";
    case ZL_ERR_CUDA: return "CUDA error";
    case ZL_ERR_OOB_BLOCK: return "block id outside the pool";
    case ZL_ERR_TIMEOUT: return "device wait timed out";
    case ZL_ERR_NCCL: return "NCCL error";
    case ZL_ERR_UNSUPPORTED: return "unsupported shape";
    case ZL_ERR_OUT_OF_BLOCKS: return "out of blocks";
    case ZL_ERR_STALE_HANDLE: return "stale handle";
    case ZL_ERR_BLOCK_NOT_ALLOCATED: return "block not allocated";
    case ZL_ERR_INVALID_BLOCK_SIZE: return "invalid block size";
    case ZL_ERR_INTERNAL: return "internal error";
    case ZL_ERR_SEQUENCE_TOO_LONG: return "sequence too long";
  }
  return "unknown status";
}

zl_status zl_ctx_create(const zl_ctx_cfg* cfg, zl_ctx** out) {
  if (!out) return set_error(ZL_ERR_INVALID_ARG, "out is null");
  *out = nullptr;
  int dev = cfg ? cfg->device : 0;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0)
    return set_error(ZL_ERR_CUDA, "no CUDA device available (%s)", cudaGetErrorString(e));
  if (dev < 0 || dev >= count)
    return set_error(ZL_ERR_INVALID_ARG, "device %d out of range (have %d)", dev, count);
  zl_ctx* ctx = new zl_ctx();
  ctx->device = dev;
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) { delete ctx; return s; }
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, dev);
  if (e != cudaSuccess) { delete ctx; return set_error(ZL_ERR_CUDA, "cudaGetDeviceProperties: %s", cudaGetErrorString(e)); }
  if (prop.major != 10) {
    delete ctx;
    return set_error(ZL_ERR_UNSUPPORTED, "libzealot_attn is built for sm_100a (B200); device %d is sm_%d%d",
                     dev, prop.major, prop.minor);
  }
  ctx->num_sms = prop.multiProcessorCount;
  // status word at [0]; the persistent prefill's two work counters at [32], a
  // 128-byte line of their own
  e = cudaMalloc(&ctx->d_status, 64 * sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_status, 0, 64 * sizeof(int));
  ctx->prefill_work = ctx->d_status + 32;
  if (e != cudaSuccess) { delete ctx; return set_error(ZL_ERR_CUDA, "status word: %s", cudaGetErrorString(e)); }
  if (cfg && cfg->workspace_bytes) {
    s = ensure_workspace(ctx, cfg->workspace_bytes);
    if (s != ZL_OK) { zl_ctx_destroy(ctx); return s; }
  }
  cudaDeviceSynchronize();
  *out = ctx;
  return ZL_OK;
}

zl_status zl_ctx_set_flags(zl_ctx* ctx, uint32_t flags) {
  if (!ctx) return set_error(ZL_ERR_INVALID_ARG, "null context");
  if (flags & ~ZL_CTX_INPUTS_AHEAD) return set_error(ZL_ERR_INVALID_ARG, "unknown context flags 0x%x", flags);
  ctx->flags = flags;
  return ZL_OK;
}

zl_status zl_nccl_finalize(zl_ctx* ctx);

zl_status zl_ctx_destroy(zl_ctx* ctx) {
  if (!ctx) return ZL_OK;
  cudaSetDevice(ctx->device);
  // First the communicator: a collective whose peer is gone is aborted (bounded
  // wait) instead of blocking the device synchronisation below for good.
  if (ctx->nccl_comm || ctx->gather_buf || ctx->nccl_done) zl_nccl_finalize(ctx);
  cudaDeviceSynchronize();
  if (ctx->d_status) cudaFree(ctx->d_status);
  if (ctx->workspace) cudaFree(ctx->workspace);
  if (ctx->counters) cudaFree(ctx->counters);
  if (ctx->activations) cudaFree(ctx->activations);
  if (ctx->sample_scratch) cudaFree(ctx->sample_scratch);
  delete ctx;
  return ZL_OK;
}

zl_status zl_check_status(zl_ctx* ctx, zl_stream stream) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  // A pending sequence-split all-gather is waited for with a deadline first, so
  // a lost peer turns into ZL_ERR_TIMEOUT here rather than a stream that never
  // drains.
  if ((s = nccl_wait_pending(ctx, ctx->nccl_timeout_ms)) != ZL_OK) return s;
  ZL_CUDA_TRY(cudaStreamSynchronize(S(stream)));
  int h = 0;
  ZL_CUDA_TRY(cudaMemcpy(&h, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost));
  ZL_CUDA_TRY(cudaMemset(ctx->d_status, 0, sizeof(int)));
  if (h && ctx->counters) {
    // A kernel that gave up may have left split-KV counters mid-count.
    ZL_CUDA_TRY(cudaMemset(ctx->counters, 0, ctx->counters_bytes));
  }
  if (h) ZL_CUDA_TRY(cudaMemset(ctx->prefill_work, 0, 2 * sizeof(int)));
  if (h & ZL_DEV_TIMEOUT) return set_error(ZL_ERR_TIMEOUT, "a bounded device wait ran out (status 0x%x)", h);
  if (h & ZL_DEV_OOB)
    return set_error(ZL_ERR_OOB_BLOCK, "a block id or slot was outside the pool (status 0x%x)", h);
  return ZL_OK;
}

uint64_t zl_launch_count(const zl_ctx* ctx) {
  return ctx ? ctx->launches.load(std::memory_order_relaxed) : 0;
}

}  // extern "C"
