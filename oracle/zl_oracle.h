/*
 * zl_oracle.h -- CPU restatement of Zealot's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA path in
 * zealot_b200/: only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline arm load it. No product code links or calls it.
 *
 * Every function restates, loop for loop and in fp32, a piece of the
 * reference Rust engine (0xnicholas/Zealot). Citations are `path:line`
 * inside that project. The reference is Rust and no Rust toolchain exists
 * on this machine, so it cannot be built and run here; the restatement is
 * pinned against the reference's own unit tests (matmul known answer,
 * repeat_interleave index mapping, attention shape / error / distinctness)
 * and otherwise follows the source line by line ("parity pinned by the
 * reference's structural tests; numeric values self-pinned by restatement").
 *
 * Arithmetic contract: fp32 everywhere, no FMA contraction (built with
 * -ffp-contract=off, as rustc does not fuse), `expf` from glibc (what Rust's
 * f32::exp calls on Linux), serial sums in the reference's loop order.
 */
#ifndef ZL_ORACLE_H
#define ZL_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GQA head -> kv head mappings used by the two reference paths. */
enum { ZLO_GQA_GROUPED = 0, /* kv = h / (H / Hkv): paged_attention.cu:32   */
       ZLO_GQA_MODULO = 1 };  /* kv = h % Hkv:       model_runner_cpu.rs:295 */

/* src/attention/mod.rs:105-115 -- c[m,n] = a[m,k] @ b[k,n], row-major,
 * accumulated in place from zero in (i, j, inner) order. */
void zlo_matmul(const float* a, const float* b, float* c, size_t m, size_t k, size_t n);

/* src/attention/mod.rs:31-103 -- CpuAttention::forward. Layout
 * [num_seqs][num_heads][max_seq_len][head_dim]; full (non-causal) softmax.
 * Returns 0, or -1 on the dimension-mismatch error of mod.rs:39-48 (the
 * caller passes each buffer's element count, as the Rust slices carry it). */
int zlo_cpu_attention_forward(const float* q, size_t q_len, const float* k, size_t k_len,
                              const float* v, size_t v_len, float* out, size_t num_seqs,
                              size_t num_heads, size_t head_dim, size_t max_seq_len);

/* src/model_runner_cpu.rs:286-304 -- [seq_len][kv_heads*d] -> [num_heads][seq_len][d],
 * q head h reads kv head h % kv_heads. */
void zlo_repeat_interleave_kv(const float* src, float* out, size_t kv_heads, size_t num_heads,
                              size_t seq_len, size_t head_dim);

/* src/model_runner_cpu.rs:172-276 -- CpuModelRunner::step for one sequence:
 * embedding gather, q/k/v projections ([in,out] weights), reshape,
 * repeat_interleave_kv, CpuAttention, last row, o-proj, lm_head.
 * logits: [vocab]. Returns 0 or -1 (attention error). */
int zlo_runner_step(const float* embedding, size_t embedding_len, const float* q_proj,
                    const float* k_proj, const float* v_proj, const float* attn_proj,
                    const float* lm_head, size_t hidden_dim, size_t num_heads,
                    size_t num_kv_heads, size_t head_dim, size_t vocab_size,
                    const int64_t* token_ids, size_t seq_len, float* logits);

/* src/kv_cache.rs:212-276 -- KVCache::store_kv: token t of [n_tokens][Hkv][d]
 * lands at pool offset block_id*bs*Hkv*d + h*bs*d + (pos%bs)*d with
 * block_id = block_ids[pos/bs], pos = start_token + t. Byte copy of
 * elem_size-byte elements (fp32 and bf16 pools alike). Returns 0, or -1 when
 * pos/bs >= n_block_ids (the OOB error of kv_cache.rs:234-239). */
int zlo_store_kv(uint8_t* k_pool, uint8_t* v_pool, const uint8_t* k, const uint8_t* v,
                 const int64_t* block_ids, size_t n_block_ids, size_t start_token,
                 size_t n_tokens, size_t num_kv_heads, size_t head_dim, size_t block_size,
                 size_t elem_size);

/* The slot-mapping form of the same scatter: slot = block_id*bs + pos%bs
 * (the per-token quantity of kv_cache.rs:241-247); slot < 0 skips the token.
 * Returns 0, or -1 when a slot is >= num_blocks*bs. */
int zlo_reshape_and_cache(uint8_t* k_pool, uint8_t* v_pool, const uint8_t* k, const uint8_t* v,
                          const int64_t* slot_mapping, size_t num_tokens, size_t num_kv_heads,
                          size_t head_dim, size_t block_size, size_t num_blocks, size_t elem_size);

/* Decode attention for one query token per sequence over its paged K/V:
 * gathers keys through the block table (a negative entry ends the sequence,
 * paged_attention.cu:66-67; the last block holds seq_len % bs tokens,
 * :69-73), then applies the CpuAttention math of mod.rs:64-97 to that single
 * query row (the last row of the reference runner, model_runner_cpu.rs:241-250).
 * q/out: [B][H][d]; pools [num_blocks][Hkv][bs][d]; fp32.
 * An empty context yields zeros. Returns 0, or -1 when a block id is >= num_blocks. */
int zlo_paged_decode(const float* q, const float* k_pool, const float* v_pool,
                     const int32_t* block_tables, const int32_t* seq_lens, float* out,
                     size_t num_seqs, size_t num_heads, size_t num_kv_heads, size_t head_dim,
                     size_t block_size, size_t max_blocks_per_seq, size_t num_blocks,
                     float scale, int gqa_map, int num_threads);

/* Same gather, restricted to tokens [tok_begin[b], tok_end[b]) of each
 * sequence, returning the unnormalised partial triple per (b, h):
 * m = max score, l = sum exp(s - m), o[d] = sum exp(s - m) * v[d].
 * Empty ranges give m = -inf, l = 0, o = 0. */
int zlo_paged_decode_partial(const float* q, const float* k_pool, const float* v_pool,
                             const int32_t* block_tables, const int32_t* tok_begin,
                             const int32_t* tok_end, float* m_out, float* l_out, float* o_out,
                             size_t num_seqs, size_t num_heads, size_t num_kv_heads,
                             size_t head_dim, size_t block_size, size_t max_blocks_per_seq,
                             size_t num_blocks, float scale, int gqa_map);

/* Merge P partial triples per row: out = sum_p e^{m_p-M} o_p / sum_p e^{m_p-M} l_p.
 * m, l: [P][rows]; o: [P][rows][d]; out: [rows][d]. */
void zlo_merge_partials(const float* m, const float* l, const float* o, float* out,
                        size_t num_parts, size_t rows, size_t head_dim);

/* Varlen prefill: packed q [T][H][d], k/v [T][Hkv][d], cu_seqlens [n+1].
 * Row i of sequence s attends to keys [0, i] (causal) or all keys of s; each
 * row is the CpuAttention row math of mod.rs:64-97, which for causal is the
 * reference runner's last row on the prefix (recompute form). */
int zlo_prefill_varlen(const float* q, const float* k, const float* v, const int32_t* cu_seqlens,
                       size_t num_seqs, float* out, size_t num_heads, size_t num_kv_heads,
                       size_t head_dim, float scale, int causal, int gqa_map, int num_threads);

/* Same, for a subset of rows only: rows listed in row_ids (global packed
 * indices), outputs packed [n_rows][H][d]. Used to sample large cases. */
int zlo_prefill_varlen_rows(const float* q, const float* k, const float* v,
                            const int32_t* cu_seqlens, size_t num_seqs, const int64_t* row_ids,
                            size_t n_rows, float* out, size_t num_heads, size_t num_kv_heads,
                            size_t head_dim, float scale, int causal, int gqa_map,
                            int num_threads);

/* src/sampling.rs:233-243 -- argmax, first maximum wins. */
int64_t zlo_argmax(const float* x, size_t n);

/* src/sampling.rs:254-273 -- softmax over finite scores (max-subtracted). */
void zlo_softmax_probs(const float* scores, float* probs, size_t n);

/* src/sampling.rs:77-230 -- Sampler::sample_with_mask with `r` the first
 * uniform draw of the rng (sampling.rs:277). mask: one byte per token (1 =
 * allowed) for tokens < mask_len, tokens >= mask_len allowed; NULL = no mask.
 * prev: previous output ids. Returns 0 (ok), 1 (EmptyLogits) or 2
 * (AllTokensMasked). *margin receives the smallest distance, at a float
 * decision that picked the token (the top-p cut, the multinomial crossing),
 * between the running sum and its threshold; +INFINITY when there is none.
 * Ties in the top-p sort, which the reference leaves to sort_unstable, are
 * broken by descending score, then ascending index. exact = 0 is the reference (f32 running sums);
 * exact = 1 evaluates the same decisions on the same f32 probabilities with
 * every sum in double (the softmax normaliser rounded to f32 once): the
 * exact-arithmetic answer the GPU sampler is held to. */
int zlo_sample(const float* logits, size_t n, const int64_t* prev, size_t n_prev, float temperature,
               uint32_t top_k, float top_p, float repetition_penalty, float frequency_penalty,
               float presence_penalty, const uint8_t* mask, size_t mask_len, float r, int exact,
               int64_t* token, float* logprob, double* margin);

/* bf16 helpers (round-to-nearest-even), used to feed the oracle exactly the
 * values a bf16 kernel sees. */
void zlo_f32_to_bf16(const float* src, uint16_t* dst, size_t n);
void zlo_bf16_to_f32(const uint16_t* src, float* dst, size_t n);

#ifdef __cplusplus
}
#endif
#endif
