/*
 * zl_oracle.c -- CPU restatement of Zealot's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernels, never part of
 * the product. See zl_oracle.h for the contract and the citation scheme
 * (`path:line` inside the reference Rust project 0xnicholas/Zealot).
 *
 * Build: gcc -O2 -ffp-contract=off -fno-fast-math -fopenmp (oracle/Makefile).
 */
#include "zl_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* src/attention/mod.rs:105-115 */
void zlo_matmul(const float* a, const float* b, float* c, size_t m, size_t k, size_t n) {
  memset(c, 0, m * n * sizeof(float));
  for (size_t i = 0; i < m; i++)
    for (size_t j = 0; j < n; j++)
      for (size_t inner = 0; inner < k; inner++) c[i * n + j] += a[i * k + inner] * b[inner * n + j];
}

/* One query row of src/attention/mod.rs:64-97, keys given as row pointers.
 * scores[] is scratch of n floats. n == 0 leaves out zeroed. */
static void attend_row(const float* q, const float* const* krow, const float* const* vrow,
                       size_t n, size_t d, float scale, float* out, float* scores) {
  if (n == 0) {
    memset(out, 0, d * sizeof(float));
    return;
  }
  for (size_t j = 0; j < n; j++) {
    float dot = 0.0f;
    for (size_t dd = 0; dd < d; dd++) dot += q[dd] * krow[j][dd];
    scores[j] = dot * scale;
  }
  float max = -INFINITY;
  for (size_t j = 0; j < n; j++) max = fmaxf(max, scores[j]);
  float sum = 0.0f;
  for (size_t j = 0; j < n; j++) sum += expf(scores[j] - max);
  for (size_t j = 0; j < n; j++) scores[j] = expf(scores[j] - max) / sum;
  for (size_t dd = 0; dd < d; dd++) {
    float acc = 0.0f;
    for (size_t j = 0; j < n; j++) acc += scores[j] * vrow[j][dd];
    out[dd] = acc;
  }
}

/* src/attention/mod.rs:31-103 */
int zlo_cpu_attention_forward(const float* q, size_t q_len, const float* k, size_t k_len,
                              const float* v, size_t v_len, float* out, size_t num_seqs,
                              size_t num_heads, size_t head_dim, size_t max_seq_len) {
  size_t expected = num_seqs * num_heads * max_seq_len * head_dim;
  if (q_len != expected || k_len != expected || v_len != expected) return -1;
  size_t n_pos = max_seq_len, d_head = head_dim;
  float scale = 1.0f / sqrtf((float)d_head);
  memset(out, 0, expected * sizeof(float));
  float* scores = (float*)malloc((n_pos * n_pos + 1) * sizeof(float));
  for (size_t s = 0; s < num_seqs; s++) {
    for (size_t h = 0; h < num_heads; h++) {
      size_t base = ((s * num_heads + h) * n_pos) * d_head;
      const float* qq = q + base;
      const float* kk = k + base;
      const float* vv = v + base;
      float* o = out + base;
      for (size_t i = 0; i < n_pos; i++)
        for (size_t j = 0; j < n_pos; j++) {
          float dot = 0.0f;
          for (size_t d = 0; d < d_head; d++) dot += qq[i * d_head + d] * kk[j * d_head + d];
          scores[i * n_pos + j] = dot * scale;
        }
      for (size_t i = 0; i < n_pos; i++) {
        float max = -INFINITY;
        for (size_t j = 0; j < n_pos; j++) max = fmaxf(max, scores[i * n_pos + j]);
        float sum = 0.0f;
        for (size_t j = 0; j < n_pos; j++) sum += expf(scores[i * n_pos + j] - max);
        for (size_t j = 0; j < n_pos; j++)
          scores[i * n_pos + j] = expf(scores[i * n_pos + j] - max) / sum;
      }
      for (size_t i = 0; i < n_pos; i++)
        for (size_t d = 0; d < d_head; d++) {
          float acc = 0.0f;
          for (size_t j = 0; j < n_pos; j++) acc += scores[i * n_pos + j] * vv[j * d_head + d];
          o[i * d_head + d] = acc;
        }
    }
  }
  free(scores);
  return 0;
}

/* src/model_runner_cpu.rs:286-304 */
void zlo_repeat_interleave_kv(const float* src, float* out, size_t kv_heads, size_t num_heads,
                              size_t seq_len, size_t head_dim) {
  for (size_t head = 0; head < num_heads; head++) {
    size_t kh = head % kv_heads;
    for (size_t pos = 0; pos < seq_len; pos++)
      for (size_t dim = 0; dim < head_dim; dim++)
        out[head * seq_len * head_dim + pos * head_dim + dim] =
            src[pos * kv_heads * head_dim + kh * head_dim + dim];
  }
}

/* src/model_runner_cpu.rs:172-276 (one sequence of the batch loop). */
int zlo_runner_step(const float* embedding, size_t embedding_len, const float* q_proj,
                    const float* k_proj, const float* v_proj, const float* attn_proj,
                    const float* lm_head, size_t hidden_dim, size_t num_heads,
                    size_t num_kv_heads, size_t head_dim, size_t vocab_size,
                    const int64_t* token_ids, size_t seq_len, float* logits) {
  size_t hid = hidden_dim, h = num_heads, d = head_dim;
  size_t kv_heads = num_kv_heads ? num_kv_heads : 1;
  size_t proj_dim = h * d, kv_proj_dim = kv_heads * d;
  float* embed_out = (float*)calloc(seq_len * hid + 1, sizeof(float));
  for (size_t i = 0; i < seq_len; i++) {
    size_t start = (size_t)token_ids[i] * hid; /* `id as usize`: negatives wrap */
    for (size_t dd = 0; dd < hid; dd++)
      embed_out[i * hid + dd] = (start + dd < embedding_len) ? embedding[start + dd] : 0.0f;
  }
  float* qp = (float*)malloc((seq_len * proj_dim + 1) * sizeof(float));
  float* kp = (float*)malloc((seq_len * kv_proj_dim + 1) * sizeof(float));
  float* vp = (float*)malloc((seq_len * kv_proj_dim + 1) * sizeof(float));
  zlo_matmul(embed_out, q_proj, qp, seq_len, hid, proj_dim);
  zlo_matmul(embed_out, k_proj, kp, seq_len, hid, kv_proj_dim);
  zlo_matmul(embed_out, v_proj, vp, seq_len, hid, kv_proj_dim);
  size_t n = h * seq_len * d;
  float* q = (float*)malloc((n + 1) * sizeof(float));
  float* k = (float*)malloc((n + 1) * sizeof(float));
  float* v = (float*)malloc((n + 1) * sizeof(float));
  float* attn_out = (float*)malloc((n + 1) * sizeof(float));
  for (size_t head = 0; head < h; head++)
    for (size_t pos = 0; pos < seq_len; pos++)
      for (size_t dim = 0; dim < d; dim++)
        q[head * seq_len * d + pos * d + dim] = qp[pos * proj_dim + head * d + dim];
  zlo_repeat_interleave_kv(kp, k, kv_heads, h, seq_len, d);
  zlo_repeat_interleave_kv(vp, v, kv_heads, h, seq_len, d);
  int rc = zlo_cpu_attention_forward(q, n, k, n, v, n, attn_out, 1, h, d, seq_len);
  if (rc == 0) {
    size_t last = seq_len ? seq_len - 1 : 0;
    float* last_hidden = (float*)calloc(hid + 1, sizeof(float));
    for (size_t head = 0; head < h; head++) {
      size_t base = head * seq_len * d + last * d;
      for (size_t dim = 0; dim < d; dim++)
        if (base + dim < n && head * d + dim < hid) last_hidden[head * d + dim] = attn_out[base + dim];
    }
    float* attn_hidden = (float*)malloc((hid + 1) * sizeof(float));
    zlo_matmul(last_hidden, attn_proj, attn_hidden, 1, hid, hid);
    zlo_matmul(attn_hidden, lm_head, logits, 1, hid, vocab_size);
    free(attn_hidden);
    free(last_hidden);
  }
  free(embed_out); free(qp); free(kp); free(vp); free(q); free(k); free(v); free(attn_out);
  return rc;
}

/* src/kv_cache.rs:212-276 */
int zlo_store_kv(uint8_t* k_pool, uint8_t* v_pool, const uint8_t* k, const uint8_t* v,
                 const int64_t* block_ids, size_t n_block_ids, size_t start_token,
                 size_t n_tokens, size_t num_kv_heads, size_t head_dim, size_t block_size,
                 size_t elem_size) {
  size_t kv_data = num_kv_heads * head_dim;
  size_t kv_block_stride = block_size * kv_data;
  for (size_t t = 0; t < n_tokens; t++) {
    size_t global_token = start_token + t;
    size_t block_idx = global_token / block_size;
    size_t token_in_block = global_token % block_size;
    if (block_idx >= n_block_ids) return -1;
    size_t block_id = (size_t)block_ids[block_idx];
    size_t src_base = t * kv_data;
    for (size_t h = 0; h < num_kv_heads; h++) {
      size_t pool_off = block_id * kv_block_stride + h * block_size * head_dim + token_in_block * head_dim;
      size_t src_off = src_base + h * head_dim;
      memcpy(k_pool + pool_off * elem_size, k + src_off * elem_size, head_dim * elem_size);
      memcpy(v_pool + pool_off * elem_size, v + src_off * elem_size, head_dim * elem_size);
    }
  }
  return 0;
}

int zlo_reshape_and_cache(uint8_t* k_pool, uint8_t* v_pool, const uint8_t* k, const uint8_t* v,
                          const int64_t* slot_mapping, size_t num_tokens, size_t num_kv_heads,
                          size_t head_dim, size_t block_size, size_t num_blocks, size_t elem_size) {
  size_t kv_data = num_kv_heads * head_dim;
  size_t kv_block_stride = block_size * kv_data;
  int rc = 0;
  for (size_t t = 0; t < num_tokens; t++) {
    int64_t slot = slot_mapping[t];
    if (slot < 0) continue;
    if ((uint64_t)slot >= (uint64_t)num_blocks * block_size) {
      rc = -1;
      continue;
    }
    size_t block_id = (size_t)slot / block_size, token_in_block = (size_t)slot % block_size;
    for (size_t h = 0; h < num_kv_heads; h++) {
      size_t pool_off = block_id * kv_block_stride + h * block_size * head_dim + token_in_block * head_dim;
      size_t src_off = t * kv_data + h * head_dim;
      memcpy(k_pool + pool_off * elem_size, k + src_off * elem_size, head_dim * elem_size);
      memcpy(v_pool + pool_off * elem_size, v + src_off * elem_size, head_dim * elem_size);
    }
  }
  return rc;
}

static size_t kv_head_of(size_t h, size_t H, size_t Hkv, int gqa_map) {
  return gqa_map == ZLO_GQA_MODULO ? h % Hkv : h / (H / Hkv);
}

/* Collects the key/value row pointers of tokens [t0, t1) of sequence b through
 * its block table; stops at a negative entry. Returns count, or -1 on an
 * out-of-pool block id. */
static long gather_rows(const float* k_pool, const float* v_pool, const int32_t* table,
                        size_t len, size_t t0, size_t t1, size_t kvh, size_t Hkv, size_t d,
                        size_t bs, size_t max_blocks, size_t num_blocks, const float** krow,
                        const float** vrow) {
  size_t nblk = (len + bs - 1) / bs;
  if (nblk > max_blocks) return -1;
  long n = 0;
  for (size_t t = 0; t < nblk; t++) {
    int32_t blk = table[t];
    if (blk < 0) break;
    if ((size_t)blk >= num_blocks) return -1;
    size_t ntok = (t == nblk - 1) ? len - t * bs : bs;
    for (size_t tok = 0; tok < ntok; tok++) {
      size_t pos = t * bs + tok;
      if (pos < t0 || pos >= t1) continue;
      size_t off = (((size_t)blk * Hkv + kvh) * bs + tok) * d;
      krow[n] = k_pool + off;
      vrow[n] = v_pool + off;
      n++;
    }
  }
  return n;
}

int zlo_paged_decode(const float* q, const float* k_pool, const float* v_pool,
                     const int32_t* block_tables, const int32_t* seq_lens, float* out,
                     size_t num_seqs, size_t num_heads, size_t num_kv_heads, size_t head_dim,
                     size_t block_size, size_t max_blocks_per_seq, size_t num_blocks,
                     float scale, int gqa_map, int num_threads) {
  int rc = 0;
  long total = (long)(num_seqs * num_heads);
#ifdef _OPENMP
  if (num_threads < 1) num_threads = 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(num_threads) reduction(min : rc)
#endif
  for (long bh = 0; bh < total; bh++) {
    size_t b = (size_t)bh / num_heads, h = (size_t)bh % num_heads;
    size_t len = seq_lens[b] > 0 ? (size_t)seq_lens[b] : 0;
    const float** krow = (const float**)malloc((len + 1) * sizeof(float*));
    const float** vrow = (const float**)malloc((len + 1) * sizeof(float*));
    float* scores = (float*)malloc((len + 1) * sizeof(float));
    size_t kvh = kv_head_of(h, num_heads, num_kv_heads, gqa_map);
    long n = gather_rows(k_pool, v_pool, block_tables + b * max_blocks_per_seq, len, 0, len, kvh,
                         num_kv_heads, head_dim, block_size, max_blocks_per_seq, num_blocks, krow,
                         vrow);
    float* o = out + (b * num_heads + h) * head_dim;
    if (n < 0) {
      rc = -1;
      memset(o, 0, head_dim * sizeof(float));
    } else {
      attend_row(q + (b * num_heads + h) * head_dim, krow, vrow, (size_t)n, head_dim, scale, o,
                 scores);
    }
    free(krow); free(vrow); free(scores);
  }
  (void)num_threads;
  return rc;
}

int zlo_paged_decode_partial(const float* q, const float* k_pool, const float* v_pool,
                             const int32_t* block_tables, const int32_t* tok_begin,
                             const int32_t* tok_end, float* m_out, float* l_out, float* o_out,
                             size_t num_seqs, size_t num_heads, size_t num_kv_heads,
                             size_t head_dim, size_t block_size, size_t max_blocks_per_seq,
                             size_t num_blocks, float scale, int gqa_map) {
  int rc = 0;
  for (size_t b = 0; b < num_seqs; b++) {
    size_t t1 = tok_end[b] > 0 ? (size_t)tok_end[b] : 0;
    size_t t0 = tok_begin[b] > 0 ? (size_t)tok_begin[b] : 0;
    const float** krow = (const float**)malloc((t1 + 1) * sizeof(float*));
    const float** vrow = (const float**)malloc((t1 + 1) * sizeof(float*));
    for (size_t h = 0; h < num_heads; h++) {
      size_t kvh = kv_head_of(h, num_heads, num_kv_heads, gqa_map);
      size_t row = b * num_heads + h;
      float* o = o_out + row * head_dim;
      long n = gather_rows(k_pool, v_pool, block_tables + b * max_blocks_per_seq, t1, t0, t1,
                           kvh, num_kv_heads, head_dim, block_size, max_blocks_per_seq,
                           num_blocks, krow, vrow);
      memset(o, 0, head_dim * sizeof(float));
      m_out[row] = -INFINITY;
      l_out[row] = 0.0f;
      if (n < 0) { rc = -1; continue; }
      if (n == 0) continue;
      const float* qq = q + row * head_dim;
      float* s = (float*)malloc((size_t)n * sizeof(float));
      float max = -INFINITY;
      for (long j = 0; j < n; j++) {
        float dot = 0.0f;
        for (size_t dd = 0; dd < head_dim; dd++) dot += qq[dd] * krow[j][dd];
        s[j] = dot * scale;
        max = fmaxf(max, s[j]);
      }
      float sum = 0.0f;
      for (long j = 0; j < n; j++) {
        float p = expf(s[j] - max);
        sum += p;
        for (size_t dd = 0; dd < head_dim; dd++) o[dd] += p * vrow[j][dd];
      }
      m_out[row] = max;
      l_out[row] = sum;
      free(s);
    }
    free(krow); free(vrow);
  }
  return rc;
}

void zlo_merge_partials(const float* m, const float* l, const float* o, float* out,
                        size_t num_parts, size_t rows, size_t head_dim) {
  for (size_t r = 0; r < rows; r++) {
    float M = -INFINITY;
    for (size_t p = 0; p < num_parts; p++) M = fmaxf(M, m[p * rows + r]);
    float* dst = out + r * head_dim;
    memset(dst, 0, head_dim * sizeof(float));
    if (M == -INFINITY) continue;
    float wsum = 0.0f;
    for (size_t p = 0; p < num_parts; p++) {
      float w = expf(m[p * rows + r] - M);
      wsum += w * l[p * rows + r];
      for (size_t dd = 0; dd < head_dim; dd++) dst[dd] += w * o[(p * rows + r) * head_dim + dd];
    }
    for (size_t dd = 0; dd < head_dim; dd++) dst[dd] /= wsum;
  }
}

static int prefill_row(const float* q, const float* k, const float* v, const int32_t* cu,
                       size_t num_seqs, size_t row, size_t H, size_t Hkv, size_t d, float scale,
                       int causal, int gqa_map, float* out_row /* [H][d] */) {
  /* locate the sequence holding packed row `row` */
  size_t s = 0;
  while (s < num_seqs && (size_t)cu[s + 1] <= row) s++;
  if (s == num_seqs) return -1;
  size_t start = (size_t)cu[s], end = (size_t)cu[s + 1];
  size_t i = row - start;
  size_t n = causal ? i + 1 : end - start;
  const float** krow = (const float**)malloc((n + 1) * sizeof(float*));
  const float** vrow = (const float**)malloc((n + 1) * sizeof(float*));
  float* scores = (float*)malloc((n + 1) * sizeof(float));
  for (size_t h = 0; h < H; h++) {
    size_t kvh = kv_head_of(h, H, Hkv, gqa_map);
    for (size_t j = 0; j < n; j++) {
      krow[j] = k + ((start + j) * Hkv + kvh) * d;
      vrow[j] = v + ((start + j) * Hkv + kvh) * d;
    }
    attend_row(q + (row * H + h) * d, krow, vrow, n, d, scale, out_row + h * d, scores);
  }
  free(krow); free(vrow); free(scores);
  return 0;
}

int zlo_prefill_varlen(const float* q, const float* k, const float* v, const int32_t* cu_seqlens,
                       size_t num_seqs, float* out, size_t num_heads, size_t num_kv_heads,
                       size_t head_dim, float scale, int causal, int gqa_map, int num_threads) {
  long total = num_seqs ? (long)cu_seqlens[num_seqs] : 0;
  int rc = 0;
#ifdef _OPENMP
  if (num_threads < 1) num_threads = 1;
#pragma omp parallel for schedule(dynamic, 4) num_threads(num_threads) reduction(min : rc)
#endif
  for (long r = 0; r < total; r++) {
    int e = prefill_row(q, k, v, cu_seqlens, num_seqs, (size_t)r, num_heads, num_kv_heads,
                        head_dim, scale, causal, gqa_map, out + (size_t)r * num_heads * head_dim);
    if (e) rc = e;
  }
  (void)num_threads;
  return rc;
}

int zlo_prefill_varlen_rows(const float* q, const float* k, const float* v,
                            const int32_t* cu_seqlens, size_t num_seqs, const int64_t* row_ids,
                            size_t n_rows, float* out, size_t num_heads, size_t num_kv_heads,
                            size_t head_dim, float scale, int causal, int gqa_map,
                            int num_threads) {
  int rc = 0;
#ifdef _OPENMP
  if (num_threads < 1) num_threads = 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(num_threads) reduction(min : rc)
#endif
  for (long r = 0; r < (long)n_rows; r++) {
    int e = prefill_row(q, k, v, cu_seqlens, num_seqs, (size_t)row_ids[r], num_heads,
                        num_kv_heads, head_dim, scale, causal, gqa_map,
                        out + (size_t)r * num_heads * head_dim);
    if (e) rc = e;
  }
  (void)num_threads;
  return rc;
}

/* src/sampling.rs:233-243 */
int64_t zlo_argmax(const float* x, size_t n) {
  int64_t best_idx = 0;
  float best_val = -INFINITY;
  for (size_t i = 0; i < n; i++)
    if (x[i] > best_val) {
      best_val = x[i];
      best_idx = (int64_t)i;
    }
  return best_idx;
}

/* ---- sampling (src/sampling.rs) ---- */

typedef struct {
  float v; /* probability */
  float s; /* score */
  size_t i;
} zlo_vi;

/* partial_cmp(..).unwrap_or(Equal), descending (sampling.rs:170-172) */
static int cmp_desc_value(const void* a, const void* b) {
  const float x = *(const float*)a, y = *(const float*)b;
  return (y > x) - (y < x);
}
/* descending probability; equal probabilities (left to sort_unstable by the
 * reference) by descending score, then ascending index */
static int cmp_desc_vi(const void* a, const void* b) {
  const zlo_vi* x = (const zlo_vi*)a;
  const zlo_vi* y = (const zlo_vi*)b;
  if (y->v > x->v) return 1;
  if (y->v < x->v) return -1;
  if (y->s > x->s) return 1;
  if (y->s < x->s) return -1;
  return (x->i > y->i) - (x->i < y->i);
}
static int cmp_i64(const void* a, const void* b) {
  const int64_t x = *(const int64_t*)a, y = *(const int64_t*)b;
  return (x > y) - (x < y);
}

/* softmax (sampling.rs:254-273). exact: the sum in double, rounded to f32 once. */
static void zlo_softmax(const float* s, float* p, size_t n, int exact) {
  float max = -INFINITY;
  for (size_t i = 0; i < n; i++)
    if (isfinite(s[i])) max = fmaxf(max, s[i]);
  float sum = 0.f;
  double dsum = 0.0;
  for (size_t i = 0; i < n; i++) {
    p[i] = isfinite(s[i]) ? expf(s[i] - max) : 0.f;
    sum += p[i];
    dsum += p[i];
  }
  if (exact) sum = (float)dsum;
  if (sum > 0.f)
    for (size_t i = 0; i < n; i++) p[i] /= sum;
}

void zlo_softmax_probs(const float* scores, float* probs, size_t n) { zlo_softmax(scores, probs, n, 0); }

int zlo_sample(const float* logits, size_t n, const int64_t* prev, size_t n_prev, float temperature,
               uint32_t top_k, float top_p, float repetition_penalty, float frequency_penalty,
               float presence_penalty, const uint8_t* mask, size_t mask_len, float r, int exact,
               int64_t* token, float* logprob, double* margin) {
  *margin = INFINITY;
  if (n == 0) return 1;
  float* s = (float*)malloc(n * sizeof(float));
  float* probs = (float*)malloc(n * sizeof(float));
  memcpy(s, logits, n * sizeof(float));
  int rc = 0;
  /* 0. constraint mask (:88-100) */
  if (mask) {
    int any = 0;
    for (size_t i = 0; i < n; i++) {
      if (i < mask_len && !mask[i]) s[i] = -INFINITY;
      any |= isfinite(s[i]);
    }
    if (!any) { rc = 2; goto out; }
  }
  /* 1. greedy (:103-110) with lightweight_logprob (:246-251) */
  if (temperature < 1e-7f) {
    const int64_t idx = zlo_argmax(s, n);
    float max = -INFINITY;
    for (size_t i = 0; i < n; i++) max = fmaxf(max, s[i]);
    float sum = 0.f;
    double dsum = 0.0;
    for (size_t i = 0; i < n; i++) {
      sum += expf(s[i] - max);
      dsum += expf(s[i] - max);
    }
    if (exact) sum = (float)dsum;
    *token = idx;
    *logprob = logf(expf(s[idx] - max) / sum);
    goto out;
  }
  /* 2. temperature (:114-119) */
  if (temperature != 1.0f) {
    const float inv_t = 1.0f / temperature;
    for (size_t i = 0; i < n; i++) s[i] *= inv_t;
  }
  /* 3/4. presence + frequency penalties from the frequency map (:125-145) */
  if ((presence_penalty != 0.f || frequency_penalty != 0.f) && n_prev > 0) {
    int64_t* ids = (int64_t*)malloc(n_prev * sizeof(int64_t));
    memcpy(ids, prev, n_prev * sizeof(int64_t));
    qsort(ids, n_prev, sizeof(int64_t), cmp_i64);
    for (size_t a = 0; a < n_prev;) {
      size_t b = a;
      while (b < n_prev && ids[b] == ids[a]) b++;
      const int64_t id = ids[a];
      const uint32_t count = (uint32_t)(b - a);
      if (id >= 0 && (uint64_t)id < n) {
        s[id] -= (float)count * frequency_penalty;
        if (presence_penalty != 0.f) s[id] -= presence_penalty;
      }
      a = b;
    }
    free(ids);
  }
  /* 5. repetition penalty, per occurrence (:148-160) */
  if (repetition_penalty != 1.0f && n_prev > 0) {
    for (size_t j = 0; j < n_prev; j++) {
      const int64_t id = prev[j];
      if (id < 0 || (uint64_t)id >= n) continue;
      if (s[id] > 0.f) s[id] /= repetition_penalty;
      else s[id] *= repetition_penalty;
    }
  }
  /* 6. top-k (:163-180) */
  if (top_k > 0) {
    const size_t k = top_k < n ? top_k : n;
    if (k < n) {
      float* sorted = (float*)malloc(n * sizeof(float));
      memcpy(sorted, s, n * sizeof(float));
      qsort(sorted, n, sizeof(float), cmp_desc_value);
      const float thr = sorted[k - 1];
      free(sorted);
      for (size_t i = 0; i < n; i++)
        if (s[i] < thr) s[i] = -INFINITY;
    }
  }
  /* 7. top-p (:183-210) */
  if (top_p > 0.f && top_p < 1.0f) {
    zlo_softmax(s, probs, n, exact);
    zlo_vi* idx = (zlo_vi*)malloc(n * sizeof(zlo_vi));
    for (size_t i = 0; i < n; i++) { idx[i].v = probs[i]; idx[i].s = s[i]; idx[i].i = i; }
    qsort(idx, n, sizeof(zlo_vi), cmp_desc_vi);
    double cum = 0.0; /* f32 accumulation unless exact */
    size_t selected = 0;
    for (size_t j = 0; j < n; j++) {
      const double before = cum;
      cum = exact ? cum + (double)idx[j].v : (double)((float)cum + idx[j].v);
      selected++;
      if (cum >= (double)top_p) {
        double m1 = fabs((double)cum - (double)top_p), m2 = fabs((double)top_p - (double)before);
        *margin = fmin(*margin, fmin(m1, m2));
        break;
      }
    }
    for (size_t j = selected; j < n; j++) s[idx[j].i] = -INFINITY;
    free(idx);
  }
  /* 8-9. softmax, all-masked check (:213-219) */
  zlo_softmax(s, probs, n, exact);
  {
    float sum = 0.f;
    for (size_t i = 0; i < n; i++) sum += probs[i];
    if (sum == 0.f || !isfinite(sum)) { rc = 2; goto out; }
  }
  /* 10. multinomial (:275-290) */
  {
    double cumsum = 0.0; /* f32 accumulation unless exact */
    size_t pick = n - 1;
    for (size_t i = 0; i < n; i++) {
      const double before = cumsum;
      cumsum = exact ? cumsum + (double)probs[i] : (double)((float)cumsum + probs[i]);
      if ((double)r < cumsum) {
        pick = i;
        *margin = fmin(*margin, fmin(fabs((double)cumsum - r), fabs((double)r - before)));
        break;
      }
    }
    *token = (int64_t)pick;
    *logprob = logf(probs[pick]);
  }
out:
  free(s);
  free(probs);
  return rc;
}

void zlo_f32_to_bf16(const float* src, uint16_t* dst, size_t n) {
  for (size_t i = 0; i < n; i++) {
    uint32_t u;
    memcpy(&u, &src[i], 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) {
      dst[i] = 0x7fc0;
      continue;
    }
    u += 0x7fffu + ((u >> 16) & 1u);
    dst[i] = (uint16_t)(u >> 16);
  }
}

void zlo_bf16_to_f32(const uint16_t* src, float* dst, size_t n) {
  for (size_t i = 0; i < n; i++) {
    uint32_t u = (uint32_t)src[i] << 16;
    memcpy(&dst[i], &u, 4);
  }
}
