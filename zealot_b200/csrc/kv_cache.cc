// kv_cache.cc -- device KV cache with the reference KVCache semantics
// (src/kv_cache.rs:51-357): per-layer K/V pools [num_blocks][Hkv][bs][d],
// per-sequence device block tables of int32 with -1 sentinels, blocks taken
// from a BlockManager. store_kv / append_kv turn the reference's per-(token,
// head) device copies into one reshape_and_cache launch per call.
#include <string>
#include <unordered_map>
#include <vector>

#include "zl_internal.h"

namespace {
struct SeqKvState {
  int32_t* d_table = nullptr;         // [max_blocks], -1 sentinels
  std::vector<uint64_t> block_ids;    // host copy, allocation order
  uint64_t cached_tokens = 0;
  int block_offset = 0;
  int max_blocks = 0;
};
}  // namespace

struct zl_kv_cache {
  zl_ctx* ctx = nullptr;
  uint64_t num_blocks = 0;
  int block_size = 0, num_layers = 0, num_kv_heads = 0, head_dim = 0;
  zl_dtype dtype = ZL_F32;
  std::vector<void*> k_pools, v_pools;
  std::unordered_map<std::string, SeqKvState> seqs;
  int64_t* d_slots = nullptr;
  size_t slots_cap = 0;
};

using namespace zl;

static zl_status unknown_seq(const char* id) {
  return set_error(ZL_ERR_INTERNAL, "KVCache: unknown seq %s", id ? id : "(null)");
}

static zl_status scatter(zl_kv_cache* kv, int layer, const void* k, const void* v,
                         const std::vector<int64_t>& slots, zl_stream stream) {
  if (slots.empty()) return ZL_OK;
  cudaStream_t st = S(stream);
  if (slots.size() > kv->slots_cap) {
    if (kv->d_slots) {
      ZL_CUDA_TRY(cudaStreamSynchronize(st));
      ZL_CUDA_TRY(cudaFree(kv->d_slots));
      kv->d_slots = nullptr;
    }
    kv->slots_cap = slots.size() * 2;
    ZL_CUDA_TRY(cudaMalloc(&kv->d_slots, kv->slots_cap * sizeof(int64_t)));
  }
  ZL_CUDA_TRY(cudaMemcpyAsync(kv->d_slots, slots.data(), slots.size() * sizeof(int64_t),
                              cudaMemcpyHostToDevice, st));
  // pageable source: the copy is staged before return, but keep ordering simple
  ZL_CUDA_TRY(cudaStreamSynchronize(st));
  return zl_reshape_and_cache(kv->ctx, k, v, kv->k_pools[layer], kv->v_pools[layer], kv->d_slots,
                              (int64_t)slots.size(), kv->num_kv_heads, kv->head_dim,
                              kv->block_size, (int64_t)kv->num_blocks, kv->dtype, stream);
}

extern "C" {

zl_status zl_kv_cache_create(zl_ctx* ctx, uint64_t num_blocks, int block_size, int num_layers,
                             int num_kv_heads, int head_dim, zl_dtype dtype, zl_kv_cache** out) {
  if (!out) return set_error(ZL_ERR_INVALID_ARG, "out is null");
  *out = nullptr;
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  if (block_size <= 0) return set_error(ZL_ERR_INVALID_BLOCK_SIZE, "Invalid block size: %d", block_size);
  if (num_layers <= 0 || num_kv_heads <= 0 || head_dim <= 0 || !dtype_ok(dtype))
    return set_error(ZL_ERR_INVALID_ARG, "KVCache: bad shape");
  auto* kv = new zl_kv_cache();
  kv->ctx = ctx;
  kv->num_blocks = num_blocks;
  kv->block_size = block_size;
  kv->num_layers = num_layers;
  kv->num_kv_heads = num_kv_heads;
  kv->head_dim = head_dim;
  kv->dtype = dtype;
  const size_t bytes = (size_t)num_blocks * block_size * num_kv_heads * head_dim * dtype_size(dtype);
  for (int l = 0; l < num_layers; l++) {
    void *kp = nullptr, *vp = nullptr;
    cudaError_t e = cudaMalloc(&kp, bytes ? bytes : 16);
    if (e == cudaSuccess) e = cudaMalloc(&vp, bytes ? bytes : 16);
    if (e == cudaSuccess) e = cudaMemset(kp, 0, bytes);  // alloc_zeros (kv_cache.rs:79-88)
    if (e == cudaSuccess) e = cudaMemset(vp, 0, bytes);
    kv->k_pools.push_back(kp);
    kv->v_pools.push_back(vp);
    if (e != cudaSuccess) {
      zl_kv_cache_destroy(kv);
      return set_error(ZL_ERR_CUDA, "KVCache pool alloc: %s", cudaGetErrorString(e));
    }
  }
  *out = kv;
  return ZL_OK;
}

zl_status zl_kv_cache_destroy(zl_kv_cache* kv) {
  if (!kv) return ZL_OK;
  cudaSetDevice(kv->ctx->device);
  cudaDeviceSynchronize();
  for (auto& it : kv->seqs) cudaFree(it.second.d_table);
  for (void* p : kv->k_pools) cudaFree(p);
  for (void* p : kv->v_pools) cudaFree(p);
  if (kv->d_slots) cudaFree(kv->d_slots);
  delete kv;
  return ZL_OK;
}

zl_status zl_kv_cache_register_seq(zl_kv_cache* kv, const char* id, int max_blocks) {
  if (!kv || !id || max_blocks < 0) return set_error(ZL_ERR_INVALID_ARG, "register_seq: bad argument");
  zl_status s = bind_device(kv->ctx);
  if (s != ZL_OK) return s;
  auto old = kv->seqs.find(id);
  if (old != kv->seqs.end()) {  // HashMap::insert replaces the previous state
    cudaFree(old->second.d_table);
    kv->seqs.erase(old);
  }
  SeqKvState st;
  st.max_blocks = max_blocks;
  std::vector<int32_t> table(max_blocks > 0 ? max_blocks : 1, -1);
  ZL_CUDA_TRY(cudaMalloc(&st.d_table, table.size() * sizeof(int32_t)));
  ZL_CUDA_TRY(cudaMemcpy(st.d_table, table.data(), table.size() * sizeof(int32_t), cudaMemcpyHostToDevice));
  kv->seqs.emplace(id, std::move(st));
  return ZL_OK;
}

zl_status zl_kv_cache_alloc_block(zl_kv_cache* kv, const char* id, zl_block_manager* bm,
                                  zl_block_handle* handle_out) {
  if (!kv || !id || !bm) return set_error(ZL_ERR_INVALID_ARG, "alloc_block: null argument");
  auto it = kv->seqs.find(id);
  if (it == kv->seqs.end()) return unknown_seq(id);
  SeqKvState& st = it->second;
  if ((int)st.block_ids.size() >= st.max_blocks)
    return set_error(ZL_ERR_INTERNAL, "block_table slice oob");
  zl_block_handle h;
  zl_status s = zl_block_manager_try_allocate(bm, &h);
  if (s != ZL_OK) return s;
  if (h.block_id >= kv->num_blocks) {
    zl_block_manager_try_free(bm, &h);
    return set_error(ZL_ERR_INTERNAL, "block %llu outside the %llu-block pool",
                     (unsigned long long)h.block_id, (unsigned long long)kv->num_blocks);
  }
  s = bind_device(kv->ctx);
  if (s != ZL_OK) return s;
  const int32_t val = (int32_t)h.block_id;
  ZL_CUDA_TRY(cudaMemcpy(st.d_table + st.block_ids.size(), &val, sizeof(int32_t), cudaMemcpyHostToDevice));
  st.block_ids.push_back(h.block_id);
  if (handle_out) *handle_out = h;
  return ZL_OK;
}

zl_status zl_kv_cache_release_seq(zl_kv_cache* kv, const char* id) {
  if (!kv || !id) return ZL_OK;
  auto it = kv->seqs.find(id);
  if (it == kv->seqs.end()) return ZL_OK;
  cudaSetDevice(kv->ctx->device);
  cudaFree(it->second.d_table);
  kv->seqs.erase(it);
  return ZL_OK;
}

zl_status zl_kv_cache_store_kv(zl_kv_cache* kv, int layer, const char* id, const void* k,
                               const void* v, uint64_t start_token, uint64_t n_tokens,
                               zl_stream stream) {
  if (!kv || !id) return set_error(ZL_ERR_INVALID_ARG, "store_kv: null argument");
  if (layer < 0 || layer >= kv->num_layers) return set_error(ZL_ERR_INVALID_ARG, "store_kv: bad layer %d", layer);
  auto it = kv->seqs.find(id);
  if (it == kv->seqs.end()) return unknown_seq(id);
  const SeqKvState& st = it->second;
  std::vector<int64_t> slots(n_tokens);
  for (uint64_t t = 0; t < n_tokens; t++) {  // kv_cache.rs:229-241
    const uint64_t g = start_token + t;
    const uint64_t bi = g / kv->block_size;
    if (bi >= st.block_ids.size())
      return set_error(ZL_ERR_INTERNAL, "KVCache store_kv: block_idx %llu OOB (have %zu blocks)",
                       (unsigned long long)bi, st.block_ids.size());
    slots[t] = (int64_t)(st.block_ids[bi] * kv->block_size + g % kv->block_size);
  }
  zl_status s = bind_device(kv->ctx);
  if (s != ZL_OK) return s;
  return scatter(kv, layer, k, v, slots, stream);
}

zl_status zl_kv_cache_append_kv(zl_kv_cache* kv, int layer, const char* id, const void* k,
                                const void* v, zl_stream stream) {
  if (!kv || !id) return set_error(ZL_ERR_INVALID_ARG, "append_kv: null argument");
  if (layer < 0 || layer >= kv->num_layers) return set_error(ZL_ERR_INVALID_ARG, "append_kv: bad layer %d", layer);
  auto it = kv->seqs.find(id);
  if (it == kv->seqs.end()) return unknown_seq(id);
  SeqKvState& st = it->second;
  const uint64_t bi = st.cached_tokens / kv->block_size;  // kv_cache.rs:304-312
  if (bi >= st.block_ids.size())
    return set_error(ZL_ERR_INTERNAL, "KVCache append_kv: block_idx %llu OOB (have %zu blocks)",
                     (unsigned long long)bi, st.block_ids.size());
  std::vector<int64_t> slots(1, (int64_t)(st.block_ids[bi] * kv->block_size + st.block_offset));
  zl_status s = bind_device(kv->ctx);
  if (s != ZL_OK) return s;
  s = scatter(kv, layer, k, v, slots, stream);
  if (s != ZL_OK) return s;
  st.cached_tokens += 1;  // kv_cache.rs:346-354
  st.block_offset += 1;
  if (st.block_offset >= kv->block_size) st.block_offset = 0;
  return ZL_OK;
}

zl_status zl_kv_cache_cached_tokens(const zl_kv_cache* kv, const char* id, uint64_t* out) {
  if (!kv || !id || !out) return set_error(ZL_ERR_INVALID_ARG, "cached_tokens: null argument");
  auto it = kv->seqs.find(id);
  if (it == kv->seqs.end()) return unknown_seq(id);
  *out = it->second.cached_tokens;
  return ZL_OK;
}

const int32_t* zl_kv_cache_block_table_ptr(const zl_kv_cache* kv, const char* id) {
  if (!kv || !id) return nullptr;
  auto it = kv->seqs.find(id);
  return it == kv->seqs.end() ? nullptr : it->second.d_table;
}

void* zl_kv_cache_k_pool_ptr(const zl_kv_cache* kv, int layer) {
  return (kv && layer >= 0 && layer < kv->num_layers) ? kv->k_pools[layer] : nullptr;
}

void* zl_kv_cache_v_pool_ptr(const zl_kv_cache* kv, int layer) {
  return (kv && layer >= 0 && layer < kv->num_layers) ? kv->v_pools[layer] : nullptr;
}

}  // extern "C"
