// ops.cu -- argument checking and kernel selection for the attention entry
// points of include/zealot_attn.h.
#include "zl_internal.h"
#include "zl_ptx.cuh"

using namespace zl;

namespace {

zl_status check_heads(int H, int Hkv, int d, const char* who) {
  if (H <= 0 || Hkv <= 0 || d <= 0)
    return set_error(ZL_ERR_INVALID_ARG, "%s: bad head shape H=%d Hkv=%d d=%d", who, H, Hkv, d);
  if (H % Hkv != 0)
    return set_error(ZL_ERR_INVALID_ARG, "%s: num_heads %d not a multiple of num_kv_heads %d", who, H, Hkv);
  return ZL_OK;
}

// One warp waits on an mbarrier whose phase never completes (count 1, no
// arrival): the bounded wait times out and flags the status word, then a
// second wait returns at once because the flag is set. Both waits end on their
// own; nothing traps.
__global__ void selftest_wait_timeout_kernel(int* status) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = zl::ptx::smem_u32(&bar);
  if (threadIdx.x == 0) {
    zl::ptx::mbar_init(b, 1);
    zl::ptx::fence_mbar_init();
  }
  __syncwarp();
  (void)zl::ptx::mbar_wait_warp(b, 0, status);  // gives up after the wait budget
  (void)zl::ptx::mbar_wait_warp(b, 0, status);  // gives up at once: the status says timed out
}

}  // namespace

extern "C" {

zl_status zl_selftest_wait_timeout(zl_ctx* ctx, zl_stream stream) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  selftest_wait_timeout_kernel<<<1, 32, 0, S(stream)>>>(ctx->d_status);
  ZL_LAUNCH_CHECK(ctx);
  return ZL_OK;
}


zl_status zl_paged_decode(zl_ctx* ctx, const void* q, const void* k_pool, const void* v_pool,
                          const int32_t* block_tables, const int32_t* seq_lens, void* out,
                          int num_seqs, int num_heads, int num_kv_heads, int head_dim,
                          int block_size, int max_blocks_per_seq, int64_t num_blocks, float scale,
                          zl_gqa_map gqa_map, int num_splits, zl_dtype dtype, zl_stream stream) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  if (!dtype_ok(dtype)) return set_error(ZL_ERR_INVALID_ARG, "paged_decode: bad dtype");
  if ((s = check_heads(num_heads, num_kv_heads, head_dim, "paged_decode")) != ZL_OK) return s;
  if (num_seqs < 0 || block_size <= 0 || max_blocks_per_seq < 0 || num_blocks < 0)
    return set_error(ZL_ERR_INVALID_ARG, "paged_decode: bad sizes B=%d bs=%d max_blocks=%d",
                     num_seqs, block_size, max_blocks_per_seq);
  if (num_seqs == 0) return ZL_OK;
  if (!q || !k_pool || !v_pool || !block_tables || !seq_lens || !out)
    return set_error(ZL_ERR_INVALID_ARG, "paged_decode: null pointer");
  const float sc = resolve_scale(scale, head_dim);
  cudaStream_t st = S(stream);
  if (dtype == ZL_BF16) {
    s = launch_decode_bf16_fast(ctx, q, k_pool, v_pool, block_tables, seq_lens, nullptr, out,
                                nullptr, nullptr, nullptr, num_seqs, num_heads, num_kv_heads,
                                head_dim, block_size, max_blocks_per_seq, num_blocks, sc, gqa_map,
                                num_splits, st);
    if (s != ZL_ERR_UNSUPPORTED) return s;
  }
  return launch_decode_generic(ctx, q, k_pool, v_pool, block_tables, seq_lens, nullptr, out,
                               nullptr, nullptr, nullptr, num_seqs, num_heads, num_kv_heads,
                               head_dim, block_size, max_blocks_per_seq, num_blocks, sc, gqa_map,
                               dtype, st);
}

zl_status zl_paged_decode_partial(zl_ctx* ctx, const void* q, const void* k_pool,
                                  const void* v_pool, const int32_t* block_tables,
                                  const int32_t* tok_begin, const int32_t* tok_end, float* m,
                                  float* l, float* o, int num_seqs, int num_heads,
                                  int num_kv_heads, int head_dim, int block_size,
                                  int max_blocks_per_seq, int64_t num_blocks, float scale,
                                  zl_gqa_map gqa_map, zl_dtype dtype, zl_stream stream) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  if (!dtype_ok(dtype)) return set_error(ZL_ERR_INVALID_ARG, "paged_decode_partial: bad dtype");
  if ((s = check_heads(num_heads, num_kv_heads, head_dim, "paged_decode_partial")) != ZL_OK) return s;
  if (num_seqs < 0 || block_size <= 0 || max_blocks_per_seq < 0 || num_blocks < 0)
    return set_error(ZL_ERR_INVALID_ARG, "paged_decode_partial: bad sizes");
  if (num_seqs == 0) return ZL_OK;
  if (!q || !k_pool || !v_pool || !block_tables || !tok_end || !m || !l || !o)
    return set_error(ZL_ERR_INVALID_ARG, "paged_decode_partial: null pointer");
  if (dtype == ZL_BF16) {
    s = launch_decode_bf16_fast(ctx, q, k_pool, v_pool, block_tables, tok_end, tok_begin, nullptr,
                                m, l, o, num_seqs, num_heads, num_kv_heads, head_dim, block_size,
                                max_blocks_per_seq, num_blocks, resolve_scale(scale, head_dim),
                                gqa_map, 0, S(stream));
    if (s != ZL_ERR_UNSUPPORTED) return s;
  }
  return launch_decode_generic(ctx, q, k_pool, v_pool, block_tables, tok_end, tok_begin, nullptr,
                               m, l, o, num_seqs, num_heads, num_kv_heads, head_dim, block_size,
                               max_blocks_per_seq, num_blocks, resolve_scale(scale, head_dim),
                               gqa_map, dtype, S(stream));
}

zl_status zl_merge_partials(zl_ctx* ctx, const float* m, const float* l, const float* o,
                            int num_parts, int64_t rows, int head_dim, void* out, zl_dtype dtype,
                            zl_stream stream) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  if (!dtype_ok(dtype) || num_parts <= 0 || rows < 0 || head_dim <= 0)
    return set_error(ZL_ERR_INVALID_ARG, "merge_partials: bad arguments");
  if (rows == 0) return ZL_OK;
  if (!m || !l || !o || !out) return set_error(ZL_ERR_INVALID_ARG, "merge_partials: null pointer");
  return launch_merge(ctx, m, l, o, num_parts, rows, head_dim, out, dtype, S(stream));
}

zl_status zl_prefill_varlen(zl_ctx* ctx, const void* q, const void* k, const void* v,
                            const int32_t* cu_seqlens, int num_seqs, int max_seq_len,
                            int64_t total_tokens, void* out,
                            int num_heads, int num_kv_heads, int head_dim, float scale, int causal,
                            zl_gqa_map gqa_map, zl_dtype dtype, zl_stream stream) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  if (!dtype_ok(dtype)) return set_error(ZL_ERR_INVALID_ARG, "prefill_varlen: bad dtype");
  if ((s = check_heads(num_heads, num_kv_heads, head_dim, "prefill_varlen")) != ZL_OK) return s;
  if (num_seqs < 0 || max_seq_len < 0 || total_tokens < 0)
    return set_error(ZL_ERR_INVALID_ARG, "prefill_varlen: bad sizes");
  if (num_seqs == 0 || max_seq_len == 0 || total_tokens == 0) return ZL_OK;
  if (!q || !k || !v || !cu_seqlens || !out)
    return set_error(ZL_ERR_INVALID_ARG, "prefill_varlen: null pointer");
  const float sc = resolve_scale(scale, head_dim);
  cudaStream_t st = S(stream);
  if (dtype == ZL_BF16) {
    s = launch_prefill_tc(ctx, q, k, v, cu_seqlens, num_seqs, max_seq_len, total_tokens, out, num_heads,
                          num_kv_heads, head_dim, sc, causal, gqa_map, st);
    if (s != ZL_ERR_UNSUPPORTED) return s;
  }
  return launch_prefill_generic(ctx, q, k, v, cu_seqlens, num_seqs, max_seq_len, total_tokens, out, num_heads,
                                num_kv_heads, head_dim, sc, causal, gqa_map, dtype, st);
}

}  // extern "C"
