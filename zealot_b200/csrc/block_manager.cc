// block_manager.cc -- restatement of the reference BlockManager
// (src/block_manager.rs:41-165): LIFO free list, refcounts, per-block
// generation starting at 1, stale-handle detection. Host-only bookkeeping;
// its block ids index the KV pools.
#include <mutex>
#include <vector>

#include "zl_internal.h"

struct zl_block_manager {
  uint64_t num_gpu_blocks = 0;
  uint64_t block_size = 0;
  std::mutex mu;
  std::vector<uint64_t> free_list;  // pop from the back
  std::vector<uint64_t> refcount;
  std::vector<uint64_t> generation;
};

using namespace zl;

static zl_status check_handle(const zl_block_manager* bm, const zl_block_handle* h) {
  // block_manager.rs:151-164
  if (h->block_id >= bm->num_gpu_blocks)
    return set_error(ZL_ERR_BLOCK_NOT_ALLOCATED, "Block %llu is not allocated",
                     (unsigned long long)h->block_id);
  const uint64_t cur = bm->generation[h->block_id];
  if (h->generation != cur)
    return set_error(ZL_ERR_STALE_HANDLE,
                     "Stale handle: block %llu was freed (gen %llu, current %llu)",
                     (unsigned long long)h->block_id, (unsigned long long)h->generation,
                     (unsigned long long)cur);
  return ZL_OK;
}

extern "C" {

zl_status zl_block_manager_create(uint64_t num_gpu_blocks, uint64_t block_size,
                                  zl_block_manager** out) {
  if (!out) return set_error(ZL_ERR_INVALID_ARG, "out is null");
  *out = nullptr;
  if (block_size == 0)  // block_manager.rs:89-91
    return set_error(ZL_ERR_INVALID_BLOCK_SIZE, "Invalid block size: %llu",
                     (unsigned long long)block_size);
  auto* bm = new zl_block_manager();
  bm->num_gpu_blocks = num_gpu_blocks;
  bm->block_size = block_size;
  bm->free_list.resize(num_gpu_blocks);
  // (0..n).collect() reversed: popping from the back yields 0, 1, 2, ...
  for (uint64_t i = 0; i < num_gpu_blocks; i++) bm->free_list[i] = num_gpu_blocks - 1 - i;
  bm->refcount.assign(num_gpu_blocks, 0);
  bm->generation.assign(num_gpu_blocks, 1);
  *out = bm;
  return ZL_OK;
}

zl_status zl_block_manager_destroy(zl_block_manager* bm) {
  delete bm;
  return ZL_OK;
}

zl_status zl_block_manager_try_allocate(zl_block_manager* bm, zl_block_handle* out) {
  if (!bm || !out) return set_error(ZL_ERR_INVALID_ARG, "null argument");
  std::lock_guard<std::mutex> g(bm->mu);
  if (bm->free_list.empty())
    return set_error(ZL_ERR_OUT_OF_BLOCKS, "Out of blocks: requested 1, available 0");
  const uint64_t id = bm->free_list.back();
  bm->free_list.pop_back();
  bm->refcount[id] = 1;
  out->block_id = id;
  out->generation = bm->generation[id];
  return ZL_OK;
}

zl_status zl_block_manager_try_free(zl_block_manager* bm, const zl_block_handle* h) {
  if (!bm || !h) return set_error(ZL_ERR_INVALID_ARG, "null argument");
  std::lock_guard<std::mutex> g(bm->mu);
  zl_status s = check_handle(bm, h);
  if (s != ZL_OK) return s;
  const uint64_t prev = bm->refcount[h->block_id];
  bm->refcount[h->block_id] = prev - 1;  // AtomicUsize::fetch_sub wraps the same way
  if (prev == 1) {
    bm->generation[h->block_id] += 1;
    bm->free_list.push_back(h->block_id);
  }
  return ZL_OK;
}

zl_status zl_block_manager_try_reference(zl_block_manager* bm, const zl_block_handle* h) {
  if (!bm || !h) return set_error(ZL_ERR_INVALID_ARG, "null argument");
  std::lock_guard<std::mutex> g(bm->mu);
  zl_status s = check_handle(bm, h);
  if (s != ZL_OK) return s;
  bm->refcount[h->block_id] += 1;
  return ZL_OK;
}

uint64_t zl_block_manager_available(const zl_block_manager* bm) {
  if (!bm) return 0;
  std::lock_guard<std::mutex> g(const_cast<zl_block_manager*>(bm)->mu);
  return bm->free_list.size();
}

}  // extern "C"
