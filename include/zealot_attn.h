/*
 * zealot_attn.h -- C ABI of libzealot_attn.so, the B200 (sm_100a) attention
 * hot path of the Zealot inference engine.
 *
 * This is the FFI surface a Rust `CudaModelRunner` (src/cuda_runner.rs,
 * src/gpu_context.rs, src/kv_cache.rs, src/attention/ of 0xnicholas/Zealot)
 * binds with `extern "C"`. Every entry point names the reference interface it
 * replaces as `path:line` inside that project.
 *
 * Conventions
 *  - Plain pointers and sizes only; device pointers are marked `device`;
 *    the caller owns every device buffer (as the reference launchers never own
 *    theirs, src/attention/cuda.rs:56-66,126-140). The library owns only the
 *    opaque zl_ctx (split-KV workspace, tensor-map cache, NCCL communicator).
 *  - Every launch takes an explicit stream (`zl_stream` = cudaStream_t; NULL
 *    is the legacy default stream) and is asynchronous.
 *  - One zl_ctx is driven from one host thread at a time, like the
 *    reference GpuContext (src/gpu_context.rs:23-26).
 *  - Errors: every call returns zl_status; zl_last_error() gives a
 *    thread-local message. Kernels never trap: a bad block id or a timed-out
 *    device wait sets a bit in the context's device status word and the kernel
 *    skips the access; zl_check_status() synchronises the stream and reports it.
 *  - There is no CPU fallback: without a CUDA device the calls return
 *    ZL_ERR_CUDA.
 */
#ifndef ZEALOT_ATTN_H
#define ZEALOT_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZL_ABI_VERSION 1

/* Status codes. The ZL_ERR_* values from OUT_OF_BLOCKS on mirror the
 * ZealotError variants of src/error.rs:4-47; a Rust wrapper maps the others
 * to ZealotError::Internal(zl_last_error()). */
typedef enum {
  ZL_OK = 0,
  ZL_ERR_INVALID_ARG = 1,        /* bad size / pointer / unsupported combination */
  ZL_ERR_CUDA = 2,               /* a CUDA runtime call failed (message has the name) */
  ZL_ERR_OOB_BLOCK = 3,          /* device: block id or slot outside the pool */
  ZL_ERR_TIMEOUT = 4,            /* device: a bounded wait ran out */
  ZL_ERR_NCCL = 5,               /* an NCCL call failed or NCCL is not loadable */
  ZL_ERR_UNSUPPORTED = 6,        /* shape the build has no kernel for */
  ZL_ERR_OUT_OF_BLOCKS = 7,      /* ZealotError::OutOfBlocks        (error.rs:11-12) */
  ZL_ERR_STALE_HANDLE = 8,       /* ZealotError::StaleHandle        (error.rs:23-28) */
  ZL_ERR_BLOCK_NOT_ALLOCATED = 9,/* ZealotError::BlockNotAllocated  (error.rs:8-9)   */
  ZL_ERR_INVALID_BLOCK_SIZE = 10,/* ZealotError::InvalidBlockSize   (error.rs:14-15) */
  ZL_ERR_INTERNAL = 11,          /* ZealotError::Internal           (error.rs:45-46) */
  ZL_ERR_SEQUENCE_TOO_LONG = 12  /* ZealotError::SequenceTooLong    (error.rs:36-37) */
} zl_status;

typedef enum { ZL_F32 = 0, ZL_BF16 = 1 } zl_dtype;

/* Query head -> KV head. GROUPED is the HF/Llama convention used by the
 * reference CUDA kernel (paged_attention.cu:32); MODULO is the CPU runner's
 * repeat_interleave_kv (model_runner_cpu.rs:295). Equal for MHA. */
typedef enum { ZL_GQA_GROUPED = 0, ZL_GQA_MODULO = 1 } zl_gqa_map;

typedef void* zl_stream;
typedef struct zl_ctx zl_ctx;

typedef struct {
  int device;                 /* CUDA ordinal */
  size_t workspace_bytes;     /* initial split-KV workspace; 0 = grow on demand */
} zl_ctx_cfg;

/* ----------------------------------------------------------------- context */

/* Replaces GpuContext::new (src/gpu_context.rs:30-52): binds a device and
 * creates the library state. cfg may be NULL (device 0). A context is used
 * from one host thread at a time (as gpu_context.rs:23-26), and its kernels
 * share its workspace and counters (split-KV partials and merge counts of the
 * decode, the persistent prefill's work counter): calls on one context whose
 * kernels may run at the same time on different streams race. Use one
 * context per stream that runs attention concurrently with another. */
zl_status zl_ctx_create(const zl_ctx_cfg* cfg, zl_ctx** out);
zl_status zl_ctx_destroy(zl_ctx* ctx);
/* Context flags (zl_ctx_set_flags). No reference counterpart.
 * ZL_CTX_INPUTS_AHEAD: the block tables, seq_lens and token ranges passed to
 * decode calls on this context are written (e.g. copied from the host) before
 * the kernel that precedes the decode on its stream starts. The decode kernel
 * is launched with programmatic stream serialization in any case -- its CTAs
 * may become resident while that kernel finishes -- and with this flag it
 * also scans the lengths and reads its first table entries before waiting for
 * that kernel; q, the pools and every output are touched only after the wait.
 * Leave it off when the preceding kernel writes the tables or lengths (a
 * device-side block-table update). */
#define ZL_CTX_INPUTS_AHEAD 1u
zl_status zl_ctx_set_flags(zl_ctx* ctx, uint32_t flags);
/* Thread-local text of the last error returned on this thread. */
const char* zl_last_error(void);
const char* zl_status_string(zl_status s);
int zl_abi_version(void);
/* Synchronises `stream`, reads and clears the device status word, returns the
 * first device-side error (ZL_ERR_OOB_BLOCK / ZL_ERR_TIMEOUT) or ZL_OK. */
zl_status zl_check_status(zl_ctx* ctx, zl_stream stream);
/* Number of kernels this context has launched (for launch accounting). */
uint64_t zl_launch_count(const zl_ctx* ctx);
/* Diagnostic, no counterpart in the reference: one warp waits on a barrier that
 * nothing completes, the way every kernel of this library waits on its
 * barriers; the bounded wait gives up after about a second, sets the timeout
 * bit of the status word and returns, and a second wait in the same warp then
 * gives up at once. The next zl_check_status reports ZL_ERR_TIMEOUT and clears
 * the word; the context stays usable. Exercises the timeout path without
 * faulting or hanging the GPU. Costs about one second of GPU time. */
zl_status zl_selftest_wait_timeout(zl_ctx* ctx, zl_stream stream);

/* ------------------------------------------------------- reshape_and_cache */

/* Replaces KVCache::store_kv / append_kv (src/kv_cache.rs:212-357), which
 * issued 2*T*Hkv device-to-device copies, with one kernel. Token t of
 * k/v [T][Hkv][d] goes to slot s = slot_mapping[t] of the pools
 * [num_blocks][Hkv][block_size][d] at element offset
 *   (s / bs)*bs*Hkv*d + h*bs*d + (s % bs)*d          (kv_cache.rs:245-247).
 * slot < 0 skips the token; slot >= num_blocks*bs sets ZL_ERR_OOB_BLOCK in
 * the status word and skips it. Bit-exact byte copy. */
zl_status zl_reshape_and_cache(zl_ctx* ctx, const void* k /*device*/, const void* v /*device*/,
                               void* k_pool /*device*/, void* v_pool /*device*/,
                               const int64_t* slot_mapping /*device*/, int64_t num_tokens,
                               int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                               zl_dtype dtype, zl_stream stream);

/* ------------------------------------------------------------ paged decode */

/* Replaces CudaAttention::paged_forward (src/attention/cuda.rs:126-210) and
 * its kernels paged_attention_kernel / paged_attention_gqa_kernel
 * (paged_attention.cu:13-291): same argument set (q/out [B][H][d], pools
 * [num_blocks][Hkv][bs][d], block_tables [B][max_blocks_per_seq] int32 with
 * negative entries ending a sequence, seq_lens [B]) plus the pool size for
 * bounds checks, the softmax scale (<= 0 means 1/sqrt(d)), the head mapping
 * and the split-KV count (0 = automatic). q, pools and out share `dtype`.
 * An empty context writes zeros. head_dim up to 256; larger head dims return
 * ZL_ERR_UNSUPPORTED. */
zl_status zl_paged_decode(zl_ctx* ctx, const void* q, const void* k_pool, const void* v_pool,
                          const int32_t* block_tables, const int32_t* seq_lens, void* out,
                          int num_seqs, int num_heads, int num_kv_heads, int head_dim,
                          int block_size, int max_blocks_per_seq, int64_t num_blocks, float scale,
                          zl_gqa_map gqa_map, int num_splits, zl_dtype dtype, zl_stream stream);

/* Allocation-free paged decode. No counterpart in the reference: it exists
 * for callers that cannot allocate device memory while they serve -- an
 * engine that hands (nearly) all HBM to its KV-cache pool at start-up has
 * nothing left for the on-demand workspace zl_paged_decode grows with
 * cudaMalloc, and a step loop that must not stall cannot take the
 * device-wide synchronisation cudaMalloc/cudaFree imply. Same kernel and
 * results as zl_paged_decode for bf16, head_dim 128, block_size 16, grouped
 * GQA with <= 8 query heads per kv head; no zl_ctx, the current device is
 * used. Its split-KV scratch is a static device array of about 5.4 MB that
 * every GPU which loads the library holds until the process exits. Limits:
 * num_seqs <= 4096 and num_seqs * num_kv_heads <= 16384, else
 * ZL_ERR_INVALID_ARG; other shapes return ZL_ERR_UNSUPPORTED. Every call
 * looks up the array's device address (no allocation); the first call on a
 * device also sets the kernel's shared-memory limit, so make that first call
 * before any stream capture. Do not carry the library across a device reset
 * without calling it again outside a capture. All calls share the array:
 * calls whose kernels overlap on the GPU race and give wrong results; calls
 * ordered on one stream are safe.
 * status (device int, required, cleared by the caller): the return code only
 * says the kernel was queued. The kernel ORs 1 (a block id or seq_len outside
 * the pool or table: that access was skipped) and 2 (a bounded wait ran out)
 * into *status. While bit 2 is set a call still returns ZL_OK but its kernel
 * does no work and leaves `out` as it was. So read and clear *status after
 * every call (or every step) before trusting `out`. */
zl_status zl_paged_decode_noalloc(const void* q, const void* k_pool, const void* v_pool,
                                  const int32_t* block_tables, const int32_t* seq_lens, void* out,
                                  int* status, int num_seqs, int num_heads, int num_kv_heads,
                                  int head_dim, int block_size, int max_blocks_per_seq,
                                  int64_t num_blocks, float scale, zl_stream stream);

/* Sequence-split form (one sequence's KV spread over GPUs): attends only to
 * tokens [tok_begin[b], tok_end[b]) of each sequence (tok_begin may be NULL =
 * 0) and writes the unnormalised partial triple per (b, h):
 *   m [B][H] = max score, l [B][H] = sum e^(s-m), o [B][H][d] = sum e^(s-m) v,
 * all fp32. Empty ranges give (-inf, 0, 0). No reference counterpart: the
 * reference has no multi-GPU path; this is the north-star sequence split. */
zl_status zl_paged_decode_partial(zl_ctx* ctx, const void* q, const void* k_pool,
                                  const void* v_pool, const int32_t* block_tables,
                                  const int32_t* tok_begin, const int32_t* tok_end, float* m,
                                  float* l, float* o, int num_seqs, int num_heads,
                                  int num_kv_heads, int head_dim, int block_size,
                                  int max_blocks_per_seq, int64_t num_blocks, float scale,
                                  zl_gqa_map gqa_map, zl_dtype dtype, zl_stream stream);

/* Merges P partial triples: out[r] = sum_p e^(m_p - M) o_p / sum_p e^(m_p - M) l_p
 * with m, l [P][rows], o [P][rows][d] fp32 and out [rows][d] in `dtype`. */
zl_status zl_merge_partials(zl_ctx* ctx, const float* m, const float* l, const float* o,
                            int num_parts, int64_t rows, int head_dim, void* out, zl_dtype dtype,
                            zl_stream stream);

/* ---------------------------------------------------------- varlen prefill */

/* Replaces CudaAttention::forward_gpu (src/attention/cuda.rs:56-110) and
 * tiled_attention_kernel (attention.cu:9-187). Packed varlen layout instead of
 * one [H][L][d] sequence: q/out [T][H][d], k/v [T][Hkv][d], cu_seqlens
 * [num_seqs+1] int32 (device) with cu_seqlens[num_seqs] == total_tokens == T
 * (the row count of the buffers, which bounds every tile load); max_seq_len
 * bounds the launch. causal != 0 masks keys after the query. bf16 with
 * head_dim 128 and an even GQA group runs on the tcgen05/TMEM tensor-core
 * kernel; other shapes on the CUDA-core kernel, head_dim up to 256 (larger:
 * ZL_ERR_UNSUPPORTED). */
zl_status zl_prefill_varlen(zl_ctx* ctx, const void* q, const void* k, const void* v,
                            const int32_t* cu_seqlens, int num_seqs, int max_seq_len,
                            int64_t total_tokens, void* out,
                            int num_heads, int num_kv_heads, int head_dim, float scale, int causal,
                            zl_gqa_map gqa_map, zl_dtype dtype, zl_stream stream);

/* ----------------------------------------------------- multi-GPU (NCCL) */

/* NCCL is loaded at run time (dlopen libnccl.so.2), so the library has no
 * link-time NCCL dependency. No reference counterpart (the reference has no
 * multi-GPU code); these carry the north-star sequence-split merge. */
zl_status zl_nccl_get_unique_id(uint8_t id_out[128]);
/* Creates a non-blocking communicator (every rank calls it with the same id)
 * and sizes the gather buffer once for steps of up to max_rows rows of up to
 * max_head_dim: nranks * max_rows * (2 + max_head_dim) fp32 of device memory.
 * timeout_ms bounds every later wait on a collective (creation gets ten times
 * that); a collective not finished by then means a peer is gone. */
zl_status zl_nccl_init(zl_ctx* ctx, const uint8_t id[128], int nranks, int rank, int64_t max_rows,
                       int max_head_dim, int timeout_ms);
/* All-gathers every rank's partial triple (m, l [rows], o [rows][d] fp32,
 * device) into the gather buffer and merges them into out [rows][d].
 * Asynchronous; allocates nothing. rows / head_dim beyond the sizes given to
 * zl_nccl_init: ZL_ERR_INVALID_ARG. After an abort: ZL_ERR_NCCL. */
zl_status zl_nccl_merge(zl_ctx* ctx, const float* m, const float* l, const float* o,
                        int64_t rows, int head_dim, void* out, zl_dtype dtype, zl_stream stream);
/* Waits up to timeout_ms (<= 0: the zl_nccl_init timeout) for the last
 * merge's all-gather. If it does not finish in time, or NCCL reports an
 * asynchronous error, the communicator is aborted (its kernels stop) and
 * ZL_ERR_TIMEOUT / ZL_ERR_NCCL is returned; the context stays usable for
 * single-GPU calls. zl_check_status does the same wait before it synchronises
 * its stream. */
zl_status zl_nccl_wait(zl_ctx* ctx, int timeout_ms);
/* Aborts the communicator at once (e.g. when the host learns that a peer is
 * gone); later zl_nccl_merge calls return ZL_ERR_NCCL. */
zl_status zl_nccl_abort(zl_ctx* ctx);
/* Destroys the communicator (aborting it if a collective cannot finish) and
 * frees the gather buffer. */
zl_status zl_nccl_finalize(zl_ctx* ctx);

/* ------------------------------------------------------------ block manager */

/* Restatement of BlockManager (src/block_manager.rs:41-165): LIFO free list
 * (a fresh pool hands out ids 0,1,2,...), refcounts, per-block generation
 * starting at 1; a handle whose generation differs is stale. Host only. */
typedef struct zl_block_manager zl_block_manager;
typedef struct {
  uint64_t block_id;
  uint64_t generation;
} zl_block_handle; /* BlockHandle, block_manager.rs:18-24 */

zl_status zl_block_manager_create(uint64_t num_gpu_blocks, uint64_t block_size,
                                  zl_block_manager** out);          /* :88-104 */
zl_status zl_block_manager_destroy(zl_block_manager* bm);
zl_status zl_block_manager_try_allocate(zl_block_manager* bm, zl_block_handle* out); /* :108-122 */
zl_status zl_block_manager_try_free(zl_block_manager* bm, const zl_block_handle* h); /* :125-135 */
zl_status zl_block_manager_try_reference(zl_block_manager* bm, const zl_block_handle* h); /* :140-144 */
uint64_t zl_block_manager_available(const zl_block_manager* bm);    /* :147-149 */

/* --------------------------------------------------------------- KV cache */

/* Restatement of KVCache (src/kv_cache.rs:51-357) for the device: per-layer
 * K/V pools [num_blocks][Hkv][bs][d] (zero-filled), per-sequence device block
 * tables of max_blocks int32 with -1 sentinels (:107-124), blocks from a
 * BlockManager (:127-161). store_kv/append_kv build a slot mapping on the host
 * and run one reshape_and_cache launch per layer call. */
typedef struct zl_kv_cache zl_kv_cache;
zl_status zl_kv_cache_create(zl_ctx* ctx, uint64_t num_blocks, int block_size, int num_layers,
                             int num_kv_heads, int head_dim, zl_dtype dtype, zl_kv_cache** out);
zl_status zl_kv_cache_destroy(zl_kv_cache* kv);
zl_status zl_kv_cache_register_seq(zl_kv_cache* kv, const char* id, int max_blocks);   /* :107-124 */
/* Returns the whole handle (the reference returns the id only and drops the
 * handle, so its blocks could never be freed with a generation check). */
zl_status zl_kv_cache_alloc_block(zl_kv_cache* kv, const char* id, zl_block_manager* bm,
                                  zl_block_handle* handle_out);                       /* :127-161 */
zl_status zl_kv_cache_release_seq(zl_kv_cache* kv, const char* id);                  /* :164-166 */
zl_status zl_kv_cache_store_kv(zl_kv_cache* kv, int layer, const char* id, const void* k,
                               const void* v, uint64_t start_token, uint64_t n_tokens,
                               zl_stream stream);                                     /* :212-276 */
zl_status zl_kv_cache_append_kv(zl_kv_cache* kv, int layer, const char* id, const void* k,
                                const void* v, zl_stream stream);                     /* :281-357 */
zl_status zl_kv_cache_cached_tokens(const zl_kv_cache* kv, const char* id, uint64_t* out);
const int32_t* zl_kv_cache_block_table_ptr(const zl_kv_cache* kv, const char* id);    /* :191-194 */
void* zl_kv_cache_k_pool_ptr(const zl_kv_cache* kv, int layer);                       /* :197-199 */
void* zl_kv_cache_v_pool_ptr(const zl_kv_cache* kv, int layer);                       /* :202-204 */

/* ------------------------------------------------------------ model runner */

/* CudaModelRunner (src/cuda_runner.rs:271-658) with the math of the CPU
 * runner it replaces (src/model_runner_cpu.rs:172-276): layer-0 weights,
 * [in,out] row-major fp32, embedding -> q/k/v -> paged KV cache ->
 * attention -> last row -> o-proj -> lm_head -> logits. Unlike the CPU runner
 * it keeps a paged KV cache, so a decode step attends over the whole history
 * (the CPU runner's recompute form). */
typedef struct zl_runner zl_runner;
typedef struct {
  int hidden_dim, num_heads, num_kv_heads, head_dim, num_layers, vocab_size;
  uint64_t num_gpu_blocks; /* SchedulerConfig::default: 1024 (scheduler.rs:168-178) */
  int block_size;          /* 16 */
  int max_blocks_per_seq;
  zl_gqa_map gqa_map;      /* ZL_GQA_MODULO reproduces the CPU runner */
} zl_runner_cfg;

typedef struct {
  const float* embedding; /* [vocab][hidden] */
  const float* q_proj;    /* [hidden][H*d]   */
  const float* k_proj;    /* [hidden][Hkv*d] */
  const float* v_proj;    /* [hidden][Hkv*d] */
  const float* attn_proj; /* [hidden][hidden]*/
  const float* lm_head;   /* [hidden][vocab] */
} zl_runner_weights;      /* host pointers, copied at create */

/* One batch entry: what Sequence::step_input / is_prefill / prefill_pos
 * (src/scheduler.rs:88-113) give the runner. */
typedef struct {
  const char* request_id;
  const int64_t* tokens; /* host */
  int num_tokens;
  int is_prefill;
  int prefill_pos;
} zl_seq_input;

zl_status zl_runner_create(zl_ctx* ctx, const zl_runner_cfg* cfg, const zl_runner_weights* w,
                           zl_runner** out);                                  /* cuda_runner.rs:52-124 */
zl_status zl_runner_destroy(zl_runner* r);
/* ModelRunner::step (src/engine.rs:18): logits_out is host [n][vocab]. */
zl_status zl_runner_step(zl_runner* r, const zl_seq_input* batch, int n, float* logits_out);
/* ModelRunner::drop_state (src/engine.rs:22). Unknown ids are ignored. */
zl_status zl_runner_drop_state(zl_runner* r, const char* request_id);

/* ---------------------------------------------------------------------------
 * Engine step of a full decoder (the layer loop of src/cuda_runner.rs:303-607:
 * RMSNorm -> q/k/v -> paged KV -> attention -> o-proj + residual -> RMSNorm ->
 * gate/up -> silu(gate)*up -> down + residual; final RMSNorm -> lm_head on the
 * last row of each sequence), batched over every sequence of the step: one
 * GEMM per projection per layer, not one per sequence. bf16 weights and
 * activations, fp32 accumulation; RMSNorm eps as given (the reference passes
 * 1e-6). All pointers are device pointers owned by the caller.
 * ------------------------------------------------------------------------- */
typedef struct {
  const void* attn_norm;  /* [hidden] bf16                                    */
  const void* wq;         /* [H*d][hidden] bf16, torch Linear layout (out,in) */
  const void* wk;         /* [Hkv*d][hidden]                                  */
  const void* wv;         /* [Hkv*d][hidden]                                  */
  const void* wo;         /* [hidden][H*d]                                    */
  const void* mlp_norm;   /* [hidden]                                         */
  const void* w_gate_up;  /* [2*inter][hidden]: gate rows, then up rows       */
  const void* w_down;     /* [hidden][inter]                                  */
} zl_layer_weights;
/* When wk starts where wq ends and wv where wk ends (one [(H+2*Hkv)*d][hidden]
 * buffer), steps of at most 256 rows compute q, k and v with one GEMM. Steps of
 * at least 512 rows compute gate/up and silu(gate)*up with zl_linear_swiglu
 * (hidden % 64 == 0, inter % 128 == 0): gate/up is then not rounded to bf16
 * before the activation. */

typedef struct {
  int num_layers, hidden, num_heads, num_kv_heads, head_dim, intermediate;
  int64_t vocab;
  float rms_eps;
  const void* embed;              /* [vocab][hidden] bf16 */
  const zl_layer_weights* layers; /* host array [num_layers] of device pointers */
  const void* final_norm;         /* [hidden] */
  const void* lm_head;            /* [vocab][hidden] */
} zl_decoder;

/* Rows [0, prefill_tokens) are prefill chunks packed back to back (sequence i
 * is rows cu_prefill[i]..cu_prefill[i+1]; each chunk attends causally to
 * itself); rows [prefill_tokens, prefill_tokens + num_decode) are one decode
 * token per sequence, attending through its block table over seq_lens[i]
 * cached tokens (its own K/V included, written by this step). */
typedef struct {
  const int64_t* tokens;       /* [T] token ids, T = prefill_tokens + num_decode */
  const int64_t* slot_mapping; /* [T] pool slot of each row's K/V               */
  const int32_t* cu_prefill;   /* [num_prefill+1]                               */
  int num_prefill, max_prefill_len;
  int64_t prefill_tokens;
  const int32_t* block_tables; /* [num_decode][max_blocks_per_seq], -1 padded   */
  const int32_t* seq_lens;     /* [num_decode]                                  */
  int num_decode, max_blocks_per_seq;
  const int32_t* last_rows;    /* [num_last] rows whose logits are produced     */
  int num_last;
} zl_step_batch;

/* The MLP's gate/up projection with the activation fused into it:
 * out[t][i] = silu(x[t] . w[i]) * (x[t] . w[I + i]) for x [M][K], w_gate_up
 * [2I][K] (gate rows, then up rows), out [M][I], all bf16, fp32 accumulation
 * on the tcgen05 tensor cores; silu(g) * u is taken from the fp32 accumulators
 * and rounded once, and the [M][2I] gate/up product never reaches HBM.
 * Replaces the gate and up GEMMs and silu_gate_mul of the reference runner
 * (src/cuda_runner.rs:529-572, src/attention/kernels/activation.cu:4-12).
 * K % 64 == 0, I % 128 == 0 and 16-byte aligned buffers, else
 * ZL_ERR_UNSUPPORTED; M == 0 is a no-op. zl_decoder_step uses it for every
 * layer whose shapes allow it. */
zl_status zl_linear_swiglu(zl_ctx* ctx, const void* x, const void* w_gate_up, void* out, int64_t M, int K,
                           int I, zl_stream stream);

/* ---------------------------------------------------------------------------
 * Sampling on the GPU for every row of a step: Sampler::sample_with_mask
 * (src/sampling.rs:77-230) per row, plus the engine's fallback to unconstrained
 * sampling when the allowed-token mask leaves nothing (src/engine.rs:190-206)
 * and token 0 when sampling still fails (src/engine.rs:214-217).
 * ------------------------------------------------------------------------- */
typedef struct {        /* SamplingParams (src/sampling.rs:22-45); seed stays with the caller */
  float temperature;    /* 1.0 default; < 1e-7 = greedy */
  int top_k;            /* 0 = off */
  float top_p;          /* 0 = off; only 0 < top_p < 1 filters */
  float repetition_penalty, frequency_penalty, presence_penalty;
} zl_sampling_params;

enum {
  ZL_SAMPLE_ALL_MASKED = 1, /* SamplingError::AllTokensMasked: token 0, logprob -inf */
  ZL_SAMPLE_FELL_BACK = 2   /* the mask left no token; sampled without it */
};

/* All pointers are device pointers. logits [num_rows][vocab] f32; params
 * [num_rows]; allowed_bits [num_rows][ceil(mask_len/32)] (bit i = token i is
 * allowed; tokens >= mask_len are allowed, as sampling.rs:91-93) or NULL;
 * mask_rows [num_rows] (1 = the row is masked) or NULL for every row;
 * penalty_offsets [num_rows+1] into penalty_ids / penalty_counts: the distinct
 * previous output tokens of each row with their occurrence counts (NULL = no
 * history); or instead dense_counts [num_rows][vocab] int32, occurrences of
 * each token in the row's output so far, with update_dense_counts = 1 adding
 * the sampled token (the history then stays on the device from step to step);
 * uniforms [num_rows]: the caller's draw r in [0, 1) per row (the
 * reference's rng.gen_range(0.0..1.0), sampling.rs:277); fallback_unmasked:
 * apply the engine's fallback. Outputs token_ids, logprobs, row_status
 * (ZL_SAMPLE_* bits; may be NULL). vocab == 0 is EmptyLogits: ZL_ERR_INVALID_ARG. */
zl_status zl_sample(zl_ctx* ctx, const float* logits, int num_rows, int64_t vocab,
                    const zl_sampling_params* params, const uint32_t* allowed_bits,
                    const uint8_t* mask_rows, int64_t mask_len, const int32_t* penalty_offsets,
                    const int64_t* penalty_ids, const int32_t* penalty_counts, int32_t* dense_counts,
                    int update_dense_counts, const float* uniforms, int fallback_unmasked,
                    int64_t* token_ids, float* logprobs, int32_t* row_status, zl_stream stream);

/* logits: device fp32 [num_last][vocab]. k_pools / v_pools: host arrays of
 * num_layers device pools, [num_blocks][Hkv][block_size][d] bf16 each.
 * Prefill chunks start at position 0 of their sequence (no cached prefix). */
zl_status zl_decoder_step(zl_ctx* ctx, const zl_decoder* model, void* const* k_pools,
                          void* const* v_pools, int64_t num_blocks, int block_size,
                          const zl_step_batch* batch, float* logits, zl_stream stream);

/* ---------------------------------------------------------------------------
 * Device-resident decode loop replayed as one CUDA graph. No counterpart in the
 * reference, whose runner copies block tables, slot mappings and tokens to the
 * device and the logits back for every sequence of every step
 * (src/cuda_runner.rs:446,645) and samples on the host (src/engine.rs:153-228).
 * `rows` decode slots keep on the device their next token, cached length,
 * block table, sampling parameters and output-token counts. A step is one
 * graph launch: staging copy (new block ids + draws) -> slots from the device
 * tables -> zl_decoder_step (decode only) -> zl_sample (next tokens written in
 * place, counts updated) -> token ids and logprobs copied to pinned host memory.
 * Block allocation stays with the caller (BlockManager::try_allocate).
 * ------------------------------------------------------------------------- */
typedef struct zl_decode_graph zl_decode_graph;
/* use_graph = 0 issues the same launches eagerly each step (for comparison).
 * The pools and weights must outlive the graph. Every row starts inactive. */
zl_status zl_decode_graph_create(zl_ctx* ctx, const zl_decoder* model, void* const* k_pools,
                                 void* const* v_pools, int64_t num_blocks, int block_size, int rows,
                                 int max_blocks_per_seq, int use_graph, zl_decode_graph** out);
zl_status zl_decode_graph_destroy(zl_decode_graph* g);
/* Row `row` takes a sequence whose first seq_len tokens are in the pools (its
 * prefill ran through zl_decoder_step): its blocks (host, n_blocks), the token
 * the next step decodes (at position seq_len), sampling parameters, and its
 * output history so far (host, for the penalties). Waits for in-flight steps. */
zl_status zl_decode_graph_set_row(zl_decode_graph* g, int row, const int32_t* block_ids, int n_blocks,
                                  int seq_len, int64_t next_token, const zl_sampling_params* params,
                                  const int64_t* history, int n_history);
/* Makes a row inactive (a finished sequence; its blocks go back to the caller). */
zl_status zl_decode_graph_clear_row(zl_decode_graph* g, int row);
/* Rows whose next step writes the first token of a new block (from the host
 * mirror of the cached lengths; no device read). rows_out has room for `rows`.
 * ZL_ERR_SEQUENCE_TOO_LONG if a row has no table entry left. */
zl_status zl_decode_graph_rows_needing_block(const zl_decode_graph* g, int32_t* rows_out, int* n_out);
/* One step. new_blocks: host [n_new][2] (row, block id), exactly one per row
 * that needs a block; uniforms: host [rows], the draw r of each row.
 * Asynchronous on `stream` (NULL: the graph's own stream). */
zl_status zl_decode_graph_step(zl_decode_graph* g, const int32_t* new_blocks, int n_new,
                               const float* uniforms, zl_stream stream);
/* Waits for the last step; copies its tokens [rows] and logprobs [rows]
 * (optional) to host memory. */
zl_status zl_decode_graph_tokens(zl_decode_graph* g, int64_t* tokens, float* logprobs);
/* Waits for the last step; copies the logits it sampled from, host
 * [rows][vocab] fp32 (before temperature, penalties and masks). */
zl_status zl_decode_graph_logits(zl_decode_graph* g, float* logits);
/* Kernel nodes in the captured graph (0 when use_graph = 0). */
int zl_decode_graph_num_kernels(const zl_decode_graph* g);

#ifdef __cplusplus
}
#endif
#endif
