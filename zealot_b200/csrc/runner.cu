// runner.cu -- CudaModelRunner for the reference engine's ModelRunner
// boundary (src/engine.rs:15-37), computing what the CPU runner computes
// (src/model_runner_cpu.rs:172-276) but keeping a paged KV cache:
//
//   embedding gather -> q/k/v = x @ W ([in,out] row-major, layer-0 weights)
//   -> reshape_and_cache of the step's new k/v -> paged decode attention of
//   each sequence's last row over its whole cached history -> o-proj ->
//   lm_head -> logits (host).
//
// All sequences of a batch go through one launch per op. The small fp32
// GEMMs here multiply in the reference's (i, j, inner) order without FMA
// contraction, so projections are bit-identical to the CPU runner's.
#include <string>
#include <unordered_map>
#include <vector>

#include "zl_internal.h"

namespace {

__global__ void embedding_gather_kernel(const int64_t* __restrict__ ids, int64_t n,
                                        const float* __restrict__ table, int64_t vocab, int hidden,
                                        float* __restrict__ out) {
  const int64_t total = n * hidden;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / hidden;
    const int c = (int)(i - t * hidden);
    const int64_t id = ids[t];
    // embedding.get(start + d).unwrap_or(0.0): out-of-range ids read zeros
    out[i] = (id >= 0 && id < vocab) ? table[id * hidden + c] : 0.f;
  }
}

// c[m,n] = a[m,k] @ b[k,n]; one thread per output, serial inner sum.
__global__ void matmul_f32_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                  float* __restrict__ c, int64_t m, int64_t k, int64_t n) {
  const int64_t total = m * n;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = idx / n, j = idx - (idx / n) * n;
    float acc = 0.f;
    for (int64_t t = 0; t < k; t++) acc = __fadd_rn(acc, __fmul_rn(a[i * k + t], b[t * n + j]));
    c[idx] = acc;
  }
}

__global__ void gather_rows_f32_kernel(const float* __restrict__ src, const int32_t* __restrict__ rows,
                                       int64_t n, int64_t width, float* __restrict__ dst) {
  const int64_t total = n * width;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / width;
    dst[i] = src[(int64_t)rows[r] * width + (i - r * width)];
  }
}

unsigned grid_for(int64_t total, int threads, int num_sms) {
  int64_t g = (total + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

}  // namespace

namespace zl {

zl_status launch_embedding_gather(zl_ctx* ctx, const int64_t* ids, int64_t n, const float* table,
                                  int64_t vocab, int hidden, float* out, cudaStream_t st) {
  if (n == 0) return ZL_OK;
  embedding_gather_kernel<<<grid_for(n * hidden, 256, ctx->num_sms), 256, 0, st>>>(ids, n, table,
                                                                                  vocab, hidden, out);
  ZL_LAUNCH_CHECK(ctx);
  return ZL_OK;
}

zl_status launch_matmul_f32(zl_ctx* ctx, const float* a, const float* b, float* c, int64_t m,
                            int64_t k, int64_t n, cudaStream_t st) {
  if (m * n == 0) return ZL_OK;
  matmul_f32_kernel<<<grid_for(m * n, 256, ctx->num_sms), 256, 0, st>>>(a, b, c, m, k, n);
  ZL_LAUNCH_CHECK(ctx);
  return ZL_OK;
}

zl_status launch_gather_rows_f32(zl_ctx* ctx, const float* src, const int32_t* rows, int64_t n,
                                 int64_t width, float* dst, cudaStream_t st) {
  if (n * width == 0) return ZL_OK;
  gather_rows_f32_kernel<<<grid_for(n * width, 256, ctx->num_sms), 256, 0, st>>>(src, rows, n,
                                                                                 width, dst);
  ZL_LAUNCH_CHECK(ctx);
  return ZL_OK;
}

}  // namespace zl

using namespace zl;

namespace {

// Device scratch that grows to the largest step seen (replaces the
// reference BufferPool, src/buffer_pool.rs:39-60, which was flushed every step).
struct Buf {
  void* p = nullptr;
  size_t cap = 0;
  zl_status ensure(size_t bytes) {
    if (bytes <= cap) return ZL_OK;
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
    size_t b = bytes < 256 ? 256 : bytes * 2;
    ZL_CUDA_TRY(cudaMalloc(&p, b));
    cap = b;
    return ZL_OK;
  }
  template <typename T> T* as() { return reinterpret_cast<T*>(p); }
};

struct SeqState {
  std::vector<zl_block_handle> handles;
  uint64_t cached = 0;  // tokens whose K/V are in the cache
};

}  // namespace

struct zl_runner {
  zl_ctx* ctx = nullptr;
  zl_runner_cfg cfg{};
  cudaStream_t stream = nullptr;
  float *emb = nullptr, *wq = nullptr, *wk = nullptr, *wv = nullptr, *wo = nullptr, *lm = nullptr;
  zl_block_manager* bm = nullptr;
  zl_kv_cache* kv = nullptr;
  std::unordered_map<std::string, SeqState> states;
  Buf ids, slots, x, q, k, v, rows, qlast, tables, lens, attn, hidden, logits;
};

static zl_status upload(float** dst, const float* src, size_t n) {
  ZL_CUDA_TRY(cudaMalloc(dst, n * sizeof(float) + 16));
  ZL_CUDA_TRY(cudaMemcpy(*dst, src, n * sizeof(float), cudaMemcpyHostToDevice));
  return ZL_OK;
}

extern "C" {

zl_status zl_runner_destroy(zl_runner* r) {
  if (!r) return ZL_OK;
  cudaSetDevice(r->ctx->device);
  cudaDeviceSynchronize();
  for (float* p : {r->emb, r->wq, r->wk, r->wv, r->wo, r->lm})
    if (p) cudaFree(p);
  for (Buf* b : {&r->ids, &r->slots, &r->x, &r->q, &r->k, &r->v, &r->rows, &r->qlast, &r->tables,
                 &r->lens, &r->attn, &r->hidden, &r->logits})
    if (b->p) cudaFree(b->p);
  if (r->kv) zl_kv_cache_destroy(r->kv);
  if (r->bm) zl_block_manager_destroy(r->bm);
  if (r->stream) cudaStreamDestroy(r->stream);
  delete r;
  return ZL_OK;
}

zl_status zl_runner_create(zl_ctx* ctx, const zl_runner_cfg* cfg, const zl_runner_weights* w,
                           zl_runner** out) {
  if (!out || !cfg || !w) return set_error(ZL_ERR_INVALID_ARG, "runner_create: null argument");
  *out = nullptr;
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  const zl_runner_cfg& c = *cfg;
  if (c.hidden_dim <= 0 || c.num_heads <= 0 || c.head_dim <= 0 || c.vocab_size <= 0 ||
      c.block_size <= 0 || c.max_blocks_per_seq <= 0)
    return set_error(ZL_ERR_INVALID_ARG, "runner_create: bad config");
  const int hkv = c.num_kv_heads > 0 ? c.num_kv_heads : 1;
  if (c.num_heads % hkv != 0)
    return set_error(ZL_ERR_INVALID_ARG, "runner_create: num_heads %% num_kv_heads != 0");
  if (c.num_heads * c.head_dim != c.hidden_dim)
    return set_error(ZL_ERR_UNSUPPORTED, "runner_create: num_heads*head_dim must equal hidden_dim");
  auto* r = new zl_runner();
  r->ctx = ctx;
  r->cfg = c;
  r->cfg.num_kv_heads = hkv;
  const size_t hid = c.hidden_dim, H = c.num_heads, d = c.head_dim;
  if ((s = upload(&r->emb, w->embedding, (size_t)c.vocab_size * hid)) != ZL_OK ||
      (s = upload(&r->wq, w->q_proj, hid * H * d)) != ZL_OK ||
      (s = upload(&r->wk, w->k_proj, hid * hkv * d)) != ZL_OK ||
      (s = upload(&r->wv, w->v_proj, hid * hkv * d)) != ZL_OK ||
      (s = upload(&r->wo, w->attn_proj, hid * hid)) != ZL_OK ||
      (s = upload(&r->lm, w->lm_head, hid * (size_t)c.vocab_size)) != ZL_OK) {
    zl_runner_destroy(r);
    return s;
  }
  if (cudaStreamCreateWithFlags(&r->stream, cudaStreamNonBlocking) != cudaSuccess) {
    zl_runner_destroy(r);
    return set_error(ZL_ERR_CUDA, "runner stream");
  }
  if ((s = zl_block_manager_create(c.num_gpu_blocks, c.block_size, &r->bm)) != ZL_OK ||
      // The CPU runner reads only layer-0 weights (model_runner_cpu.rs:193-265),
      // so one layer of cache carries all the state its logits depend on.
      (s = zl_kv_cache_create(ctx, c.num_gpu_blocks, c.block_size, 1, hkv, c.head_dim, ZL_F32,
                              &r->kv)) != ZL_OK) {
    zl_runner_destroy(r);
    return s;
  }
  *out = r;
  return ZL_OK;
}

zl_status zl_runner_drop_state(zl_runner* r, const char* request_id) {
  if (!r || !request_id) return ZL_OK;
  auto it = r->states.find(request_id);
  if (it == r->states.end()) return ZL_OK;
  for (const zl_block_handle& h : it->second.handles) zl_block_manager_try_free(r->bm, &h);
  r->states.erase(it);
  return zl_kv_cache_release_seq(r->kv, request_id);
}

zl_status zl_runner_step(zl_runner* r, const zl_seq_input* batch, int n, float* logits_out) {
  if (!r) return set_error(ZL_ERR_INVALID_ARG, "runner_step: null runner");
  if (n == 0) return ZL_OK;
  if (n < 0 || !batch || !logits_out) return set_error(ZL_ERR_INVALID_ARG, "runner_step: bad batch");
  zl_status s = bind_device(r->ctx);
  if (s != ZL_OK) return s;
  const zl_runner_cfg& c = r->cfg;
  const int hid = c.hidden_dim, H = c.num_heads, Hkv = c.num_kv_heads, d = c.head_dim;
  const int bs = c.block_size, mb = c.max_blocks_per_seq;
  cudaStream_t st = r->stream;

  // 1. per-sequence state, blocks and slot mapping of this step's tokens
  std::vector<int64_t> ids, slots;
  std::vector<int32_t> last_rows(n), lens(n), tables((size_t)n * mb, -1);
  for (int i = 0; i < n; i++) {
    const zl_seq_input& in = batch[i];
    if (!in.request_id || in.num_tokens <= 0 || !in.tokens)
      return set_error(ZL_ERR_INVALID_ARG, "runner_step: sequence %d has no input", i);
    // A prefill from position 0 recomputes the sequence (scheduler preempt path,
    // src/scheduler.rs:374-376): its old cache is discarded.
    if (in.is_prefill && in.prefill_pos == 0) zl_runner_drop_state(r, in.request_id);
    auto it = r->states.find(in.request_id);
    if (it == r->states.end()) {
      if ((s = zl_kv_cache_register_seq(r->kv, in.request_id, mb)) != ZL_OK) return s;
      it = r->states.emplace(in.request_id, SeqState()).first;
    }
    SeqState& ss = it->second;
    const uint64_t start = ss.cached, end = start + in.num_tokens;
    const uint64_t need = (end + bs - 1) / bs;
    if (need > (uint64_t)mb)
      return set_error(ZL_ERR_SEQUENCE_TOO_LONG,
                       "Sequence too long: worst case needs %llu blocks, pool capacity is %d",
                       (unsigned long long)need, mb);
    while (ss.handles.size() < need) {
      zl_block_handle h;
      if ((s = zl_kv_cache_alloc_block(r->kv, in.request_id, r->bm, &h)) != ZL_OK) return s;
      ss.handles.push_back(h);  // freed with its generation in drop_state
    }
    for (uint64_t p = start; p < end; p++) {
      ids.push_back(in.tokens[p - start]);
      slots.push_back((int64_t)(ss.handles[p / bs].block_id * bs + p % bs));
    }
    last_rows[i] = (int32_t)(ids.size() - 1);
    lens[i] = (int32_t)end;
    for (size_t b = 0; b < ss.handles.size(); b++) tables[(size_t)i * mb + b] = (int32_t)ss.handles[b].block_id;
  }
  const int64_t T = (int64_t)ids.size();

  // 2. device buffers
  if ((s = r->ids.ensure(T * 8)) || (s = r->slots.ensure(T * 8)) || (s = r->x.ensure(T * hid * 4)) ||
      (s = r->q.ensure(T * H * d * 4)) || (s = r->k.ensure(T * Hkv * d * 4)) ||
      (s = r->v.ensure(T * Hkv * d * 4)) || (s = r->rows.ensure(n * 4)) ||
      (s = r->qlast.ensure((size_t)n * H * d * 4)) || (s = r->tables.ensure(tables.size() * 4)) ||
      (s = r->lens.ensure(n * 4)) || (s = r->attn.ensure((size_t)n * H * d * 4)) ||
      (s = r->hidden.ensure((size_t)n * hid * 4)) || (s = r->logits.ensure((size_t)n * c.vocab_size * 4)))
    return s;
  ZL_CUDA_TRY(cudaMemcpyAsync(r->ids.p, ids.data(), T * 8, cudaMemcpyHostToDevice, st));
  ZL_CUDA_TRY(cudaMemcpyAsync(r->slots.p, slots.data(), T * 8, cudaMemcpyHostToDevice, st));
  ZL_CUDA_TRY(cudaMemcpyAsync(r->rows.p, last_rows.data(), n * 4, cudaMemcpyHostToDevice, st));
  ZL_CUDA_TRY(cudaMemcpyAsync(r->tables.p, tables.data(), tables.size() * 4, cudaMemcpyHostToDevice, st));
  ZL_CUDA_TRY(cudaMemcpyAsync(r->lens.p, lens.data(), n * 4, cudaMemcpyHostToDevice, st));

  // 3. embedding + projections for every new token
  zl_ctx* ctx = r->ctx;
  if ((s = launch_embedding_gather(ctx, r->ids.as<int64_t>(), T, r->emb, c.vocab_size, hid, r->x.as<float>(), st)) ||
      (s = launch_matmul_f32(ctx, r->x.as<float>(), r->wq, r->q.as<float>(), T, hid, (int64_t)H * d, st)) ||
      (s = launch_matmul_f32(ctx, r->x.as<float>(), r->wk, r->k.as<float>(), T, hid, (int64_t)Hkv * d, st)) ||
      (s = launch_matmul_f32(ctx, r->x.as<float>(), r->wv, r->v.as<float>(), T, hid, (int64_t)Hkv * d, st)))
    return s;
  // 4. new K/V into the paged pool
  if ((s = zl_reshape_and_cache(ctx, r->k.p, r->v.p, zl_kv_cache_k_pool_ptr(r->kv, 0),
                                zl_kv_cache_v_pool_ptr(r->kv, 0), r->slots.as<int64_t>(), T, Hkv, d,
                                bs, (int64_t)c.num_gpu_blocks, ZL_F32, st)))
    return s;
  // 5. last query row of every sequence attends over its whole history
  if ((s = launch_gather_rows_f32(ctx, r->q.as<float>(), r->rows.as<int32_t>(), n, (int64_t)H * d,
                                  r->qlast.as<float>(), st)) ||
      (s = zl_paged_decode(ctx, r->qlast.p, zl_kv_cache_k_pool_ptr(r->kv, 0),
                           zl_kv_cache_v_pool_ptr(r->kv, 0), r->tables.as<int32_t>(),
                           r->lens.as<int32_t>(), r->attn.p, n, H, Hkv, d, bs, mb,
                           (int64_t)c.num_gpu_blocks, 0.f, c.gqa_map, 0, ZL_F32, st)))
    return s;
  // 6. o-proj and lm_head on the last rows ([n][H*d] == [n][hidden])
  if ((s = launch_matmul_f32(ctx, r->attn.as<float>(), r->wo, r->hidden.as<float>(), n, hid, hid, st)) ||
      (s = launch_matmul_f32(ctx, r->hidden.as<float>(), r->lm, r->logits.as<float>(), n, hid, c.vocab_size, st)))
    return s;
  ZL_CUDA_TRY(cudaMemcpyAsync(logits_out, r->logits.p, (size_t)n * c.vocab_size * 4,
                              cudaMemcpyDeviceToHost, st));
  if ((s = zl_check_status(ctx, st)) != ZL_OK) return s;
  for (int i = 0; i < n; i++) r->states[batch[i].request_id].cached += batch[i].num_tokens;
  return ZL_OK;
}

}  // extern "C"
