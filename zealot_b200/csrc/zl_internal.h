// zl_internal.h -- shared host-side state and helpers of libzealot_attn.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/zealot_attn.h"

// Bits of the per-context device status word (kernels atomicOr them).
enum : int {
  ZL_DEV_OOB = 1,      // block id / slot outside the pool, or table overflow
  ZL_DEV_TIMEOUT = 2,  // a bounded wait gave up
};

struct zl_ctx {
  int device = 0;
  uint32_t flags = 0;             // ZL_CTX_* (zl_ctx_set_flags)
  int num_sms = 148;
  int* d_status = nullptr;        // device status word
  int* prefill_work = nullptr;    // [0] next work item, [1] CTAs finished: the persistent prefill's
                                  // counters (zero between launches; in the status allocation)
  void* workspace = nullptr;      // split-KV partials + per-segment counters
  size_t workspace_bytes = 0;
  void* counters = nullptr;       // zeroed int32 counters, self-resetting
  size_t counters_bytes = 0;
  std::atomic<uint64_t> launches{0};
  // NCCL (loaded at run time)
  void* nccl_comm = nullptr;
  int nranks = 1, rank = 0;
  void* gather_buf = nullptr;     // sized once at zl_nccl_init: nranks x max_rows x (2 + max_d) fp32
  size_t gather_bytes = 0;
  int64_t nccl_max_rows = 0;
  int nccl_max_d = 0;
  int nccl_timeout_ms = 0;        // bound of zl_nccl_wait / zl_check_status on a pending collective
  cudaEvent_t nccl_done = nullptr;  // recorded after the last enqueued all-gather
  bool nccl_pending = false;      // an all-gather was enqueued and not yet seen complete
  bool nccl_aborted = false;      // the communicator was aborted (a peer was lost)
  // decoder-step activations (residual stream, q/k/v, attention out, MLP)
  void* activations = nullptr;
  size_t activation_bytes = 0;
  // sampling rows that do not fit in shared memory
  void* sample_scratch = nullptr;
  size_t sample_scratch_bytes = 0;
};

namespace zl {

zl_status set_error(zl_status s, const char* fmt, ...);
inline zl_status ok() { return ZL_OK; }

// Makes the context's device current; returns ZL_ERR_CUDA on failure.
zl_status bind_device(zl_ctx* ctx);

// Grows the context workspace (stream-ordered free of the old one is not
// needed: callers synchronise through the stream they pass).
zl_status ensure_workspace(zl_ctx* ctx, size_t bytes);
zl_status ensure_counters(zl_ctx* ctx, size_t bytes);

inline cudaStream_t S(zl_stream s) { return reinterpret_cast<cudaStream_t>(s); }

#define ZL_CUDA_TRY(expr)                                                            \
  do {                                                                               \
    cudaError_t _e = (expr);                                                         \
    if (_e != cudaSuccess)                                                           \
      return ::zl::set_error(ZL_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,            \
                             cudaGetErrorString(_e), __FILE__, __LINE__);            \
  } while (0)

#define ZL_LAUNCH_CHECK(ctx)                                                         \
  do {                                                                               \
    cudaError_t _e = cudaGetLastError();                                             \
    if (_e != cudaSuccess)                                                           \
      return ::zl::set_error(ZL_ERR_CUDA, "kernel launch failed: %s (%s:%d)",       \
                             cudaGetErrorString(_e), __FILE__, __LINE__);            \
    (ctx)->launches.fetch_add(1, std::memory_order_relaxed);                         \
  } while (0)

inline size_t dtype_size(zl_dtype t) { return t == ZL_F32 ? 4 : 2; }
inline bool dtype_ok(zl_dtype t) { return t == ZL_F32 || t == ZL_BF16; }

// Internal launchers shared between translation units.
zl_status launch_decode_generic(zl_ctx* ctx, const void* q, const void* k_pool,
                                const void* v_pool, const int32_t* block_tables,
                                const int32_t* seq_lens, const int32_t* tok_begin,
                                void* out, float* m_out, float* l_out, float* o_out,
                                int B, int H, int Hkv, int d, int bs, int max_blocks,
                                int64_t num_blocks, float scale, zl_gqa_map map,
                                zl_dtype dtype, cudaStream_t st);
// Both prefill launchers check cu_seqlens on the device against total_tokens
// (ZL_DEV_OOB and the sequence skipped when it leaves [0, total_tokens]).
zl_status launch_prefill_generic(zl_ctx* ctx, const void* q, const void* k, const void* v,
                                 const int32_t* cu_seqlens, int num_seqs, int max_seq_len,
                                 int64_t total_tokens, void* out, int H, int Hkv, int d, float scale,
                                 int causal, zl_gqa_map map, zl_dtype dtype, cudaStream_t st);
// Fast bf16 decode (paged_decode_bf16.cu). Returns ZL_ERR_UNSUPPORTED when the
// shape is outside its envelope so the caller can use the CUDA-core kernel.
// With o_out != nullptr it computes the partial triple (m_out, l_out, o_out)
// over [tok_begin[b], seq_lens[b]) instead of the normalised `out`.
zl_status launch_decode_bf16_fast(zl_ctx* ctx, const void* q, const void* k_pool,
                                  const void* v_pool, const int32_t* block_tables,
                                  const int32_t* seq_lens, const int32_t* tok_begin, void* out,
                                  float* m_out, float* l_out, float* o_out, int B, int H, int Hkv,
                                  int d, int bs, int max_blocks, int64_t num_blocks, float scale,
                                  zl_gqa_map map, int num_splits, cudaStream_t st);
zl_status launch_prefill_tc(zl_ctx* ctx, const void* q, const void* k, const void* v,
                            const int32_t* cu_seqlens, int num_seqs, int max_seq_len,
                            int64_t total_tokens, void* out,
                            int H, int Hkv, int d, float scale, int causal, zl_gqa_map map,
                            cudaStream_t st);
// Gate/up projection with the SwiGLU epilogue (gemm_swiglu.cu); ZL_ERR_UNSUPPORTED
// outside its shape envelope (K % 64, I % 128, 16-byte alignment).
zl_status launch_gemm_swiglu(zl_ctx* ctx, const void* x, const void* w, void* out, int64_t M, int K, int I,
                             cudaStream_t st);
zl_status launch_merge(zl_ctx* ctx, const float* m, const float* l, const float* o, int P,
                       int64_t rows, int d, void* out, zl_dtype dtype, cudaStream_t st);
zl_status launch_embedding_gather(zl_ctx* ctx, const int64_t* ids, int64_t n, const float* table,
                                  int64_t vocab, int hidden, float* out, cudaStream_t st);
zl_status launch_matmul_f32(zl_ctx* ctx, const float* a, const float* b, float* c, int64_t m,
                            int64_t k, int64_t n, cudaStream_t st);
zl_status launch_gather_rows_f32(zl_ctx* ctx, const float* src, const int32_t* rows, int64_t n,
                                 int64_t width, float* dst, cudaStream_t st);

// Waits (bounded by the context's NCCL timeout) for the last enqueued NCCL
// all-gather; aborts the communicator when it does not finish in time or NCCL
// reports an asynchronous error. ZL_OK when nothing is pending.
zl_status nccl_wait_pending(zl_ctx* ctx, int timeout_ms);

// Default softmax scale 1/sqrt(d) computed like src/attention/mod.rs:53.
inline float resolve_scale(float scale, int d) {
  return scale > 0.f ? scale : 1.0f / sqrtf((float)d);
}

}  // namespace zl
