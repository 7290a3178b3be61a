// reshape_and_cache.cu -- scatter new K/V rows into the paged pools.
//
// Replaces KVCache::store_kv / append_kv (src/kv_cache.rs:212-357 of the
// reference), which issued one 4*d-byte device-to-device memcpy per
// (token, kv head) and per tensor, with a single HBM-bound kernel:
// every thread moves one 16-byte chunk of K and the same chunk of V.
// Destination offset (elements), as kv_cache.rs:245-247:
//   block_id*bs*Hkv*d + h*bs*d + token_in_block*d,  block_id = slot / bs.
#include "zl_internal.h"

namespace {

__global__ void __launch_bounds__(256)
reshape_and_cache_vec16(const uint4* __restrict__ k, const uint4* __restrict__ v,
                        uint4* __restrict__ k_pool, uint4* __restrict__ v_pool,
                        const int64_t* __restrict__ slot_mapping, int64_t num_tokens, int hkv,
                        int chunks_per_head, int bs, int64_t num_slots, int* status) {
  const int64_t chunks_per_token = (int64_t)hkv * chunks_per_head;
  const int64_t total = num_tokens * chunks_per_token;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / chunks_per_token;
    const int64_t r = i - t * chunks_per_token;
    const int h = (int)(r / chunks_per_head);
    const int c = (int)(r - (int64_t)h * chunks_per_head);
    const int64_t slot = __ldg(slot_mapping + t);
    if (slot < 0) continue;
    if (slot >= num_slots) {
      if (r == 0) atomicOr(status, ZL_DEV_OOB);
      continue;
    }
    const int64_t blk = slot / bs;
    const int64_t tib = slot - blk * bs;
    const int64_t dst = ((blk * hkv + h) * bs + tib) * chunks_per_head + c;
    const uint4 kk = __ldcs(k + i);
    const uint4 vv = __ldcs(v + i);
    k_pool[dst] = kk;
    v_pool[dst] = vv;
  }
}

// Element-wise form for rows whose byte size is not a multiple of 16 or for
// unaligned pointers.
template <typename T>
__global__ void __launch_bounds__(256)
reshape_and_cache_elem(const T* __restrict__ k, const T* __restrict__ v, T* __restrict__ k_pool,
                       T* __restrict__ v_pool, const int64_t* __restrict__ slot_mapping,
                       int64_t num_tokens, int hkv, int d, int bs, int64_t num_slots, int* status) {
  const int64_t per_token = (int64_t)hkv * d;
  const int64_t total = num_tokens * per_token;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per_token;
    const int64_t r = i - t * per_token;
    const int h = (int)(r / d);
    const int e = (int)(r - (int64_t)h * d);
    const int64_t slot = slot_mapping[t];
    if (slot < 0) continue;
    if (slot >= num_slots) {
      if (r == 0) atomicOr(status, ZL_DEV_OOB);
      continue;
    }
    const int64_t blk = slot / bs;
    const int64_t tib = slot - blk * bs;
    const int64_t dst = ((blk * hkv + h) * bs + tib) * d + e;
    k_pool[dst] = k[i];
    v_pool[dst] = v[i];
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" zl_status zl_reshape_and_cache(zl_ctx* ctx, const void* k, const void* v, void* k_pool,
                                          void* v_pool, const int64_t* slot_mapping,
                                          int64_t num_tokens, int num_kv_heads, int head_dim,
                                          int block_size, int64_t num_blocks, zl_dtype dtype,
                                          zl_stream stream) {
  using namespace zl;
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  if (!dtype_ok(dtype)) return set_error(ZL_ERR_INVALID_ARG, "reshape_and_cache: bad dtype %d", (int)dtype);
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_blocks < 0)
    return set_error(ZL_ERR_INVALID_ARG,
                     "reshape_and_cache: bad sizes T=%lld Hkv=%d d=%d bs=%d blocks=%lld",
                     (long long)num_tokens, num_kv_heads, head_dim, block_size, (long long)num_blocks);
  if (num_tokens == 0) return ZL_OK;
  if (!k || !v || !k_pool || !v_pool || !slot_mapping)
    return set_error(ZL_ERR_INVALID_ARG, "reshape_and_cache: null pointer");
  const size_t es = dtype_size(dtype);
  const int64_t num_slots = num_blocks * block_size;
  cudaStream_t st = S(stream);
  const size_t row_bytes = (size_t)head_dim * es;
  const int threads = 256;
  if (row_bytes % 16 == 0 && aligned16(k) && aligned16(v) && aligned16(k_pool) && aligned16(v_pool)) {
    const int cph = (int)(row_bytes / 16);
    const int64_t total = num_tokens * num_kv_heads * cph;
    int64_t blocks = (total + threads - 1) / threads;
    const int64_t cap = (int64_t)ctx->num_sms * 32;
    if (blocks > cap) blocks = cap;
    reshape_and_cache_vec16<<<(unsigned)blocks, threads, 0, st>>>(
        (const uint4*)k, (const uint4*)v, (uint4*)k_pool, (uint4*)v_pool, slot_mapping, num_tokens,
        num_kv_heads, cph, block_size, num_slots, ctx->d_status);
  } else {
    const int64_t total = num_tokens * num_kv_heads * head_dim;
    int64_t blocks = (total + threads - 1) / threads;
    const int64_t cap = (int64_t)ctx->num_sms * 32;
    if (blocks > cap) blocks = cap;
    if (dtype == ZL_F32)
      reshape_and_cache_elem<float><<<(unsigned)blocks, threads, 0, st>>>(
          (const float*)k, (const float*)v, (float*)k_pool, (float*)v_pool, slot_mapping,
          num_tokens, num_kv_heads, head_dim, block_size, num_slots, ctx->d_status);
    else
      reshape_and_cache_elem<uint16_t><<<(unsigned)blocks, threads, 0, st>>>(
          (const uint16_t*)k, (const uint16_t*)v, (uint16_t*)k_pool, (uint16_t*)v_pool,
          slot_mapping, num_tokens, num_kv_heads, head_dim, block_size, num_slots, ctx->d_status);
  }
  ZL_LAUNCH_CHECK(ctx);
  return ZL_OK;
}
