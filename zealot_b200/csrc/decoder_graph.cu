// decoder_graph.cu -- a device-resident decode loop replayed as one CUDA graph.
//
// The reference runner copies block tables, slot mappings and token ids to the
// device and the logits back to the host for every sequence of every step
// (src/cuda_runner.rs:446 and :645), and the engine samples on the host
// (src/engine.rs:153-228). Here a fixed set of `rows` decode slots keeps on the
// device everything a decode step reads: each row's next token, its cached
// length, its block table, its sampling parameters and its output-token counts
// (for the penalties). One step is:
//
//   H2D  pinned staging -> device: new block ids (rows that cross into a new
//        16-token block) and the caller's uniform draws (two pinned staging
//        buffers, one graph each, so the host can fill step k+1's while step k
//        runs)
//   advance kernel: apply the new block ids to the device tables; for each
//        active row slot = table[len / bs] * bs + len % bs, len += 1
//   zl_decoder_step (decode rows only)  -> logits
//   zl_sample (dense counts, updated)   -> each row's next token, in place
//   D2H  token ids and logprobs -> pinned host memory
//
// captured once into a CUDA graph (or, for comparison, issued eagerly). Block
// allocation stays with the caller's BlockManager: the host mirrors the cached
// lengths, so it knows which rows need a block before the step without reading
// anything back. Rows are recycled: a finished sequence's row is cleared
// (length 0: no cache write, zero attention output) and a new sequence whose
// prefill ran through zl_decoder_step takes it over.
#include <cstring>
#include <vector>

#include "zl_internal.h"

struct zl_decode_graph {
  zl_ctx* ctx = nullptr;
  zl_decoder model{};
  std::vector<zl_layer_weights> layers;
  std::vector<void*> k_pools, v_pools;
  int64_t num_blocks = 0;
  int bs = 16, rows = 0, max_blocks = 0;
  bool use_graph = true;
  // device state
  int64_t* d_tokens = nullptr;
  int32_t* d_lens = nullptr;
  int32_t* d_tables = nullptr;
  int64_t* d_slots = nullptr;
  int32_t* d_cu = nullptr;
  int32_t* d_last = nullptr;
  float* d_logits = nullptr;
  float* d_logprobs = nullptr;
  int32_t* d_row_status = nullptr;
  zl_sampling_params* d_params = nullptr;
  int32_t* d_counts = nullptr;
  uint8_t* d_stage = nullptr;
  // pinned host
  uint8_t* h_stage[2] = {nullptr, nullptr};
  int64_t* h_tokens = nullptr;
  float* h_logprobs = nullptr;
  size_t stage_bytes = 0;
  std::vector<int32_t> h_lens;  // cached tokens per row (0 = inactive)
  cudaStream_t stream = nullptr;  // capture stream
  cudaEvent_t done[2] = {nullptr, nullptr};  // end of the last step that used staging buffer i
  cudaGraph_t graph[2] = {nullptr, nullptr};
  cudaGraphExec_t exec[2] = {nullptr, nullptr};
  int graph_kernels = 0;
  uint64_t steps = 0;
  int last = 0;  // staging buffer of the last step
};

namespace {

// staging block: header, then new-block pairs, then uniforms
struct StageHeader {
  int32_t n_new;
  int32_t pad[3];
};
__host__ __device__ inline size_t stage_blocks_off() { return sizeof(StageHeader); }
__host__ __device__ inline size_t stage_uniforms_off(int rows) { return sizeof(StageHeader) + (size_t)rows * 2 * sizeof(int32_t); }

__global__ void __launch_bounds__(1024) advance_kernel(const uint8_t* __restrict__ stage, int32_t* __restrict__ tables,
                                                        int32_t* __restrict__ lens, int64_t* __restrict__ slots,
                                                        int rows, int max_blocks, int bs, int* status) {
  const StageHeader* h = reinterpret_cast<const StageHeader*>(stage);
  const int32_t* nb = reinterpret_cast<const int32_t*>(stage + stage_blocks_off());
  const int n_new = h->n_new;
  // new blocks first: row r gets block id b at the table index of its next position
  for (int u = threadIdx.x; u < n_new; u += blockDim.x) {
    const int r = nb[2 * u], b = nb[2 * u + 1];
    if (r < 0 || r >= rows) continue;
    const int idx = lens[r] / bs;
    if (idx < max_blocks) tables[(int64_t)r * max_blocks + idx] = b;
  }
  __syncthreads();
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    const int len = lens[r];
    if (len <= 0) {
      slots[r] = -1;  // inactive row: no cache write, empty attention
      continue;
    }
    const int idx = len / bs;
    const int b = idx < max_blocks ? tables[(int64_t)r * max_blocks + idx] : -1;
    if (b < 0) {
      atomicOr(status, ZL_DEV_OOB);  // the caller did not supply the row's next block
      slots[r] = -1;
    } else {
      slots[r] = (int64_t)b * bs + len % bs;
    }
    lens[r] = len + 1;
  }
}

__global__ void iota_kernel(int32_t* p, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = i;
}

zl_status run_body(zl_decode_graph* g, int buf, cudaStream_t st) {
  using namespace zl;
  zl_ctx* ctx = g->ctx;
  ZL_CUDA_TRY(cudaMemcpyAsync(g->d_stage, g->h_stage[buf], g->stage_bytes, cudaMemcpyHostToDevice, st));
  advance_kernel<<<1, 1024, 0, st>>>(g->d_stage, g->d_tables, g->d_lens, g->d_slots, g->rows, g->max_blocks, g->bs,
                                     ctx->d_status);
  ZL_LAUNCH_CHECK(ctx);
  zl_step_batch b{};
  b.tokens = g->d_tokens;
  b.slot_mapping = g->d_slots;
  b.cu_prefill = g->d_cu;
  b.num_prefill = 0;
  b.max_prefill_len = 0;
  b.prefill_tokens = 0;
  b.block_tables = g->d_tables;
  b.seq_lens = g->d_lens;
  b.num_decode = g->rows;
  b.max_blocks_per_seq = g->max_blocks;
  b.last_rows = g->d_last;
  b.num_last = g->rows;
  zl_status s = zl_decoder_step(ctx, &g->model, g->k_pools.data(), g->v_pools.data(), g->num_blocks, g->bs, &b,
                                g->d_logits, st);
  if (s != ZL_OK) return s;
  const float* unif = reinterpret_cast<const float*>(g->d_stage + stage_uniforms_off(g->rows));
  s = zl_sample(ctx, g->d_logits, g->rows, g->model.vocab, g->d_params, nullptr, nullptr, 0, nullptr, nullptr,
                nullptr, g->d_counts, 1, unif, 1, g->d_tokens, g->d_logprobs, g->d_row_status, st);
  if (s != ZL_OK) return s;
  ZL_CUDA_TRY(cudaMemcpyAsync(g->h_tokens, g->d_tokens, (size_t)g->rows * 8, cudaMemcpyDeviceToHost, st));
  ZL_CUDA_TRY(cudaMemcpyAsync(g->h_logprobs, g->d_logprobs, (size_t)g->rows * 4, cudaMemcpyDeviceToHost, st));
  return ZL_OK;
}

}  // namespace

using namespace zl;

extern "C" zl_status zl_decode_graph_destroy(zl_decode_graph* g) {
  if (!g) return ZL_OK;
  if (g->ctx) cudaSetDevice(g->ctx->device);
  if (g->stream) cudaStreamSynchronize(g->stream);
  cudaDeviceSynchronize();
  for (int i = 0; i < 2; i++) {
    if (g->exec[i]) cudaGraphExecDestroy(g->exec[i]);
    if (g->graph[i]) cudaGraphDestroy(g->graph[i]);
    if (g->done[i]) cudaEventDestroy(g->done[i]);
    if (g->h_stage[i]) cudaFreeHost(g->h_stage[i]);
  }
  for (void* p : {(void*)g->d_tokens, (void*)g->d_lens, (void*)g->d_tables, (void*)g->d_slots, (void*)g->d_cu,
                  (void*)g->d_last, (void*)g->d_logits, (void*)g->d_logprobs, (void*)g->d_row_status,
                  (void*)g->d_params, (void*)g->d_counts, (void*)g->d_stage})
    if (p) cudaFree(p);
  for (void* p : {(void*)g->h_tokens, (void*)g->h_logprobs})
    if (p) cudaFreeHost(p);
  if (g->stream) cudaStreamDestroy(g->stream);
  delete g;
  return ZL_OK;
}

extern "C" zl_status zl_decode_graph_create(zl_ctx* ctx, const zl_decoder* model, void* const* k_pools,
                                            void* const* v_pools, int64_t num_blocks, int block_size, int rows,
                                            int max_blocks_per_seq, int use_graph, zl_decode_graph** out) {
  if (!out) return set_error(ZL_ERR_INVALID_ARG, "decode_graph_create: null out");
  *out = nullptr;
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  if (!model || !model->layers || !k_pools || !v_pools || rows <= 0 || rows > 4096 || max_blocks_per_seq <= 0 ||
      block_size <= 0 || num_blocks <= 0 || model->num_layers <= 0 || model->vocab <= 0)
    return set_error(ZL_ERR_INVALID_ARG, "decode_graph_create: bad arguments");
  auto* g = new zl_decode_graph();
  g->ctx = ctx;
  g->model = *model;
  g->layers.assign(model->layers, model->layers + model->num_layers);
  g->model.layers = g->layers.data();
  g->k_pools.assign(k_pools, k_pools + model->num_layers);
  g->v_pools.assign(v_pools, v_pools + model->num_layers);
  g->num_blocks = num_blocks;
  g->bs = block_size;
  g->rows = rows;
  g->max_blocks = max_blocks_per_seq;
  g->use_graph = use_graph != 0;
  g->h_lens.assign(rows, 0);
  g->stage_bytes = stage_uniforms_off(rows) + (size_t)rows * 4;
  const int64_t V = model->vocab;
  auto fail = [&](zl_status st) {
    zl_decode_graph_destroy(g);
    return st;
  };
#define ZG_TRY(expr)                                                                                   \
  do {                                                                                                 \
    cudaError_t _e = (expr);                                                                           \
    if (_e != cudaSuccess)                                                                             \
      return fail(set_error(ZL_ERR_CUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e),      \
                            __FILE__, __LINE__));                                                      \
  } while (0)
  ZG_TRY(cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking));
  for (int i = 0; i < 2; i++) {
    ZG_TRY(cudaEventCreateWithFlags(&g->done[i], cudaEventDisableTiming));
    ZG_TRY(cudaHostAlloc(&g->h_stage[i], g->stage_bytes, cudaHostAllocDefault));
    memset(g->h_stage[i], 0, g->stage_bytes);
  }
  ZG_TRY(cudaMalloc(&g->d_tokens, rows * 8));
  ZG_TRY(cudaMalloc(&g->d_lens, rows * 4));
  ZG_TRY(cudaMalloc(&g->d_tables, (size_t)rows * max_blocks_per_seq * 4));
  ZG_TRY(cudaMalloc(&g->d_slots, rows * 8));
  ZG_TRY(cudaMalloc(&g->d_cu, 16));
  ZG_TRY(cudaMalloc(&g->d_last, rows * 4));
  ZG_TRY(cudaMalloc(&g->d_logits, (size_t)rows * V * 4));
  ZG_TRY(cudaMalloc(&g->d_logprobs, rows * 4));
  ZG_TRY(cudaMalloc(&g->d_row_status, rows * 4));
  ZG_TRY(cudaMalloc(&g->d_params, rows * sizeof(zl_sampling_params)));
  ZG_TRY(cudaMalloc(&g->d_counts, (size_t)rows * V * 4));
  ZG_TRY(cudaMalloc(&g->d_stage, g->stage_bytes));
  ZG_TRY(cudaHostAlloc(&g->h_tokens, rows * 8, cudaHostAllocDefault));
  ZG_TRY(cudaHostAlloc(&g->h_logprobs, rows * 4, cudaHostAllocDefault));
  ZG_TRY(cudaMemset(g->d_tokens, 0, rows * 8));
  ZG_TRY(cudaMemset(g->d_lens, 0, rows * 4));
  ZG_TRY(cudaMemset(g->d_tables, 0xff, (size_t)rows * max_blocks_per_seq * 4));
  ZG_TRY(cudaMemset(g->d_cu, 0, 16));
  std::vector<zl_sampling_params> greedy(rows, zl_sampling_params{0.f, 0, 0.f, 1.f, 0.f, 0.f});
  ZG_TRY(cudaMemcpy(g->d_params, greedy.data(), rows * sizeof(zl_sampling_params), cudaMemcpyHostToDevice));
  iota_kernel<<<(rows + 255) / 256, 256, 0, g->stream>>>(g->d_last, rows);
  ZG_TRY(cudaGetLastError());
  // One eager pass (every row inactive) sizes every lazily grown buffer -- the
  // activations, the split-KV workspace and counters, shared-memory limits --
  // so that nothing allocates while the graph is captured.
  if ((s = run_body(g, 0, g->stream)) != ZL_OK) return fail(s);
  ZG_TRY(cudaStreamSynchronize(g->stream));
  if ((s = zl_check_status(ctx, g->stream)) != ZL_OK) return fail(s);
  ZG_TRY(cudaMemset(g->d_counts, 0, (size_t)rows * V * 4));
  ZG_TRY(cudaMemset(g->d_tokens, 0, rows * 8));
  if (g->use_graph) {
    const uint64_t before = ctx->launches.load();
    for (int i = 0; i < 2; i++) {
      ZG_TRY(cudaStreamBeginCapture(g->stream, cudaStreamCaptureModeThreadLocal));
      s = run_body(g, i, g->stream);
      cudaGraph_t graph = nullptr;
      const cudaError_t e = cudaStreamEndCapture(g->stream, &graph);
      if (s != ZL_OK) {
        if (graph) cudaGraphDestroy(graph);
        return fail(s);
      }
      if (e != cudaSuccess)
        return fail(set_error(ZL_ERR_CUDA, "graph capture failed: %s", cudaGetErrorString(e)));
      g->graph[i] = graph;
      ZG_TRY(cudaGraphInstantiate(&g->exec[i], graph, 0));
    }
    ctx->launches.store(before);  // captured launches ran no kernel
    size_t n = 0;
    ZG_TRY(cudaGraphGetNodes(g->graph[0], nullptr, &n));
    std::vector<cudaGraphNode_t> nodes(n);
    ZG_TRY(cudaGraphGetNodes(g->graph[0], nodes.data(), &n));
    for (cudaGraphNode_t nd : nodes) {
      cudaGraphNodeType t;
      if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) g->graph_kernels++;
    }
  }
  for (int i = 0; i < 2; i++) ZG_TRY(cudaEventRecord(g->done[i], g->stream));
  ZG_TRY(cudaStreamSynchronize(g->stream));
#undef ZG_TRY
  *out = g;
  return ZL_OK;
}

extern "C" zl_status zl_decode_graph_set_row(zl_decode_graph* g, int row, const int32_t* block_ids, int n_blocks,
                                             int seq_len, int64_t next_token, const zl_sampling_params* params,
                                             const int64_t* history, int n_history) {
  if (!g) return set_error(ZL_ERR_INVALID_ARG, "decode_graph_set_row: null graph");
  zl_status s = bind_device(g->ctx);
  if (s != ZL_OK) return s;
  if (row < 0 || row >= g->rows || seq_len <= 0 || n_blocks < 0 || n_blocks > g->max_blocks ||
      (n_blocks > 0 && !block_ids) || (int64_t)n_blocks * g->bs < seq_len || !params || n_history < 0 ||
      (n_history > 0 && !history) || next_token < 0 || next_token >= g->model.vocab)
    return set_error(ZL_ERR_INVALID_ARG, "decode_graph_set_row: bad arguments for row %d", row);
  for (int i = 0; i < n_blocks; i++)
    if (block_ids[i] < 0 || block_ids[i] >= g->num_blocks)
      return set_error(ZL_ERR_INVALID_ARG, "decode_graph_set_row: block id %d outside the pool", block_ids[i]);
  ZL_CUDA_TRY(cudaStreamSynchronize(g->stream));
  for (int i = 0; i < 2; i++) ZL_CUDA_TRY(cudaEventSynchronize(g->done[i]));
  const int64_t V = g->model.vocab;
  std::vector<int32_t> table(g->max_blocks, -1);
  for (int i = 0; i < n_blocks; i++) table[i] = block_ids[i];
  std::vector<int32_t> counts(V, 0);
  for (int i = 0; i < n_history; i++)
    if (history[i] >= 0 && history[i] < V) counts[history[i]]++;
  ZL_CUDA_TRY(cudaMemcpy(g->d_tables + (int64_t)row * g->max_blocks, table.data(), g->max_blocks * 4,
                         cudaMemcpyHostToDevice));
  ZL_CUDA_TRY(cudaMemcpy(g->d_counts + row * V, counts.data(), V * 4, cudaMemcpyHostToDevice));
  ZL_CUDA_TRY(cudaMemcpy(g->d_lens + row, &seq_len, 4, cudaMemcpyHostToDevice));
  ZL_CUDA_TRY(cudaMemcpy(g->d_tokens + row, &next_token, 8, cudaMemcpyHostToDevice));
  ZL_CUDA_TRY(cudaMemcpy(g->d_params + row, params, sizeof(zl_sampling_params), cudaMemcpyHostToDevice));
  g->h_lens[row] = seq_len;
  return ZL_OK;
}

extern "C" zl_status zl_decode_graph_clear_row(zl_decode_graph* g, int row) {
  if (!g || row < 0 || row >= g->rows) return set_error(ZL_ERR_INVALID_ARG, "decode_graph_clear_row: bad row");
  zl_status s = bind_device(g->ctx);
  if (s != ZL_OK) return s;
  ZL_CUDA_TRY(cudaStreamSynchronize(g->stream));
  for (int i = 0; i < 2; i++) ZL_CUDA_TRY(cudaEventSynchronize(g->done[i]));
  const int32_t zero = 0;
  ZL_CUDA_TRY(cudaMemcpy(g->d_lens + row, &zero, 4, cudaMemcpyHostToDevice));
  ZL_CUDA_TRY(cudaMemset(g->d_tables + (int64_t)row * g->max_blocks, 0xff, g->max_blocks * 4));
  g->h_lens[row] = 0;
  return ZL_OK;
}

extern "C" zl_status zl_decode_graph_rows_needing_block(const zl_decode_graph* g, int32_t* rows_out, int* n_out) {
  if (!g || !rows_out || !n_out) return set_error(ZL_ERR_INVALID_ARG, "decode_graph_rows_needing_block: null");
  int n = 0;
  for (int r = 0; r < g->rows; r++) {
    const int len = g->h_lens[r];
    if (len > 0 && len % g->bs == 0) {
      if (len / g->bs >= g->max_blocks)
        return set_error(ZL_ERR_SEQUENCE_TOO_LONG, "row %d: %d cached tokens fill its %d blocks", r, len,
                         g->max_blocks);
      rows_out[n++] = r;
    }
  }
  *n_out = n;
  return ZL_OK;
}

extern "C" zl_status zl_decode_graph_step(zl_decode_graph* g, const int32_t* new_blocks, int n_new,
                                          const float* uniforms, zl_stream stream) {
  if (!g || n_new < 0 || (n_new > 0 && !new_blocks) || !uniforms)
    return set_error(ZL_ERR_INVALID_ARG, "decode_graph_step: bad arguments");
  zl_status s = bind_device(g->ctx);
  if (s != ZL_OK) return s;
  // every row that enters a new block gets exactly one, inside the pool
  std::vector<char> need(g->rows, 0), got(g->rows, 0);
  for (int r = 0; r < g->rows; r++) need[r] = g->h_lens[r] > 0 && g->h_lens[r] % g->bs == 0;
  for (int u = 0; u < n_new; u++) {
    const int r = new_blocks[2 * u], b = new_blocks[2 * u + 1];
    if (r < 0 || r >= g->rows || !need[r] || got[r] || b < 0 || b >= g->num_blocks)
      return set_error(ZL_ERR_INVALID_ARG, "decode_graph_step: unexpected new block (%d, %d)", r, b);
    if (g->h_lens[r] / g->bs >= g->max_blocks)
      return set_error(ZL_ERR_SEQUENCE_TOO_LONG, "row %d has no table entry left", r);
    got[r] = 1;
  }
  for (int r = 0; r < g->rows; r++)
    if (need[r] && !got[r]) return set_error(ZL_ERR_INVALID_ARG, "decode_graph_step: row %d needs a block", r);
  // staging buffer `buf` was last read by the step two back
  const int buf = (int)(g->steps & 1);
  ZL_CUDA_TRY(cudaEventSynchronize(g->done[buf]));
  auto* h = reinterpret_cast<StageHeader*>(g->h_stage[buf]);
  h->n_new = n_new;
  if (n_new) memcpy(g->h_stage[buf] + stage_blocks_off(), new_blocks, (size_t)n_new * 8);
  memcpy(g->h_stage[buf] + stage_uniforms_off(g->rows), uniforms, (size_t)g->rows * 4);
  cudaStream_t st = stream ? S(stream) : g->stream;
  if (g->use_graph) {
    ZL_CUDA_TRY(cudaGraphLaunch(g->exec[buf], st));
  } else if ((s = run_body(g, buf, st)) != ZL_OK) {
    return s;
  }
  ZL_CUDA_TRY(cudaEventRecord(g->done[buf], st));
  g->last = buf;
  for (int r = 0; r < g->rows; r++)
    if (g->h_lens[r] > 0) g->h_lens[r]++;
  g->steps++;
  return ZL_OK;
}

extern "C" zl_status zl_decode_graph_tokens(zl_decode_graph* g, int64_t* tokens, float* logprobs) {
  if (!g || !tokens) return set_error(ZL_ERR_INVALID_ARG, "decode_graph_tokens: null");
  zl_status s = bind_device(g->ctx);
  if (s != ZL_OK) return s;
  ZL_CUDA_TRY(cudaEventSynchronize(g->done[g->last]));
  memcpy(tokens, g->h_tokens, (size_t)g->rows * 8);
  if (logprobs) memcpy(logprobs, g->h_logprobs, (size_t)g->rows * 4);
  return ZL_OK;
}

extern "C" zl_status zl_decode_graph_logits(zl_decode_graph* g, float* logits) {
  if (!g || !logits) return set_error(ZL_ERR_INVALID_ARG, "decode_graph_logits: null");
  zl_status s = bind_device(g->ctx);
  if (s != ZL_OK) return s;
  ZL_CUDA_TRY(cudaEventSynchronize(g->done[g->last]));
  ZL_CUDA_TRY(cudaMemcpy(logits, g->d_logits, (size_t)g->rows * g->model.vocab * sizeof(float),
                         cudaMemcpyDeviceToHost));
  return ZL_OK;
}

extern "C" int zl_decode_graph_num_kernels(const zl_decode_graph* g) { return g ? g->graph_kernels : 0; }
