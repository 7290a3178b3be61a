// sampling.cu -- token sampling on the GPU for a whole step: one CTA per row of
// logits, restating Sampler::sample_with_mask (src/sampling.rs:77-230) and the
// engine's fallback to unconstrained sampling when a grammar mask leaves no
// token (src/engine.rs:190-217).
//
// Pipeline per row (the reference's order):
//   0. allowed-token mask -> -inf; all masked -> AllTokensMasked   (sampling.rs:88-100)
//   1. temperature < 1e-7: greedy argmax (first maximum) + logprob  (:103-110, :233-252)
//   2. temperature scaling                                          (:114-119)
//   3/4. frequency and presence penalties per unique previous token (:125-145)
//   5. repetition penalty, once per occurrence                      (:148-160)
//   6. top-k: scores below the k-th largest -> -inf                 (:163-180)
//   7. top-p: keep the smallest descending-probability prefix whose
//      mass reaches top_p                                           (:183-210)
//   8-10. softmax, all-masked check, multinomial draw with the
//      caller's uniform r, logprob = ln p                           (:213-230, :275-290)
//
// Steps 0-6 are bit-exact float operations (no contraction). The reference sums
// probabilities serially in f32; here every sum that decides a token (the top-p
// prefix mass, the multinomial CDF) is an exact integer sum of the f32
// probabilities in 2^-40 fixed point, so the result is deterministic and equal
// to the exact-arithmetic decision; it can differ from the reference's only
// where the reference's own rounding decides (a margin of a few f32 ulps).
// Top-k and top-p thresholds come from 8-bit radix selects over order-preserving
// keys in shared memory (4 passes each), not from sorting the vocabulary.
#include <math_constants.h>

#include "zl_internal.h"

namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr double kFix = 1099511627776.0;  // 2^40
constexpr int kMaxSmemVocab = (200 * 1024) / 4;

using u64 = unsigned long long;

struct SampleArgs {
  const float* logits;
  int64_t vocab;
  const zl_sampling_params* params;
  const uint32_t* allowed;  // [n][words] bitmask, bit set = allowed
  const uint8_t* mask_rows;  // [n] 1 = row uses the mask (nullptr = every row)
  int64_t mask_len;
  int64_t mask_words;
  const int32_t* pen_off;  // [n+1]
  const int64_t* pen_ids;  // unique in-range token ids per row
  const int32_t* pen_cnt;  // occurrences of each
  int32_t* dense_counts;   // [n][vocab] occurrences per token (alternative to the lists)
  int update_counts;       // add the sampled token to dense_counts
  const float* uniforms;   // [n]
  int fallback_unmasked;
  float* scratch;          // [n][vocab] when the row does not fit in shared memory
  int64_t* token_ids;
  float* logprobs;
  int32_t* row_status;
};

struct Shared {
  uint32_t cnt[256];
  u64 mass[256];
  float rf[kWarps];
  int ri[kWarps];
  u64 ru[kWarps];
  double rd[kWarps];
  uint32_t digit;
  u64 above;
  u64 draw;
  int64_t token;
  int found;
};

__device__ __forceinline__ uint32_t ord_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ float block_max(float v, Shared& sh) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh.rf[w] = v;
  __syncthreads();
  float r = sh.rf[l];
  for (int o = 16; o; o >>= 1) r = fmaxf(r, __shfl_xor_sync(0xffffffffu, r, o));
  return r;
}

// fmaxf ignores NaN, like f32::max in the reference's folds.
__device__ __forceinline__ bool finite_f(float x) { return isfinite(x); }

__device__ double block_sum_d(double v, Shared& sh) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh.rd[w] = v;
  __syncthreads();
  double r = sh.rd[l];
  for (int o = 16; o; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}

// softmax normaliser: the sum of the f32 exponentials in double, rounded once
__device__ float softmax_sum(const float* s, int64_t V, float mx, Shared& sh) {
  double acc = 0.0;
  for (int64_t i = threadIdx.x; i < V; i += kThreads) acc += finite_f(s[i]) ? (double)expf(s[i] - mx) : 0.0;
  return (float)block_sum_d(acc, sh);
}


// Finds, over elements whose key matches (key & mask) == prefix, the 8-bit digit
// at `shift` such that counting from the top digit down, the running total first
// reaches `want`. Counts (by_mass = false) or fixed-point masses (true).
// Returns with sh.digit, and sh.above = total strictly above the digit.
__device__ void pick_digit(Shared& sh, u64 want, bool by_mass) {
  if (threadIdx.x < 32) {
    const int l = threadIdx.x;
    // lane l covers digits 255-8l .. 248-8l (descending)
    u64 v[8];
    u64 tot = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int d = 255 - 8 * l - k;
      v[k] = by_mass ? sh.mass[d] : (u64)sh.cnt[d];
      tot += v[k];
    }
    u64 incl = tot;
    for (int o = 1; o < 32; o <<= 1) {
      const u64 t = __shfl_up_sync(0xffffffffu, incl, o);
      if (l >= o) incl += t;
    }
    const u64 excl = incl - tot;
    const unsigned hit = __ballot_sync(0xffffffffu, excl < want && incl >= want);
    if (hit) {
      const int src = __ffs(hit) - 1;
      if (l == src) {
        u64 acc = excl;
#pragma unroll
        for (int k = 0; k < 8; k++) {
          if (acc + v[k] >= want) {
            sh.digit = 255 - 8 * l - k;
            sh.above = acc;
            sh.found = 1;
            break;
          }
          acc += v[k];
        }
      }
    } else if (l == 0) {
      sh.found = 0;
    }
  }
  __syncthreads();
}

// Radix histogram update for one element per lane (d = 0xffffffff: no element).
// All 32 lanes, converged. Lanes holding the same digit combine first (the keys
// of a row fall into a handful of digits in the early passes), then one lane per
// digit adds to shared memory. An element's mass is at most 2^40, so the two
// 20-bit halves of 32 lanes' masses sum within 32 bits.
__device__ __forceinline__ void hist_add(uint32_t d, u64 m, Shared& sh, bool mass) {
  const unsigned peers = __match_any_sync(0xffffffffu, d);
  if (d == 0xffffffffu) return;
  const bool leader = (int)(threadIdx.x & 31) == __ffs(peers) - 1;
  if (!mass) {
    if (leader) atomicAdd(&sh.cnt[d], (uint32_t)__popc(peers));
    return;
  }
  const uint32_t lo = __reduce_add_sync(peers, (uint32_t)(m & 0xfffffu));
  const uint32_t hi = __reduce_add_sync(peers, (uint32_t)(m >> 20));
  if (leader) {
    atomicAdd(&sh.cnt[d], (uint32_t)__popc(peers));
    atomicAdd(&sh.mass[d], ((u64)hi << 20) + lo);
  }
}

// p_i of the top-p / final softmax, as f32 like the reference, then in fixed point.
__device__ __forceinline__ float prob_of(float s, float mx, float sum) {
  return finite_f(s) ? __fdiv_rn(expf(s - mx), sum) : 0.f;
}
__device__ __forceinline__ u64 fix_of(float p) { return (u64)llrint((double)p * kFix); }

// Returns true and writes (token, logprob) on success; false = AllTokensMasked.
__device__ bool sample_row(const SampleArgs& a, const zl_sampling_params& p, int row, float* s,
                           const float* lg, bool masked, Shared& sh, int64_t& token, float& logprob) {
  const int64_t V = a.vocab;
  const int tid = threadIdx.x;
  // 0. mask
  int any_finite = 0;
  for (int64_t i = tid; i < V; i += kThreads) {
    float v = lg[i];
    if (masked && i < a.mask_len &&
        !((a.allowed[(int64_t)row * a.mask_words + (i >> 5)] >> (i & 31)) & 1u))
      v = -CUDART_INF_F;
    s[i] = v;
    any_finite |= finite_f(v);
  }
  any_finite = __syncthreads_or(any_finite);
  if (masked && !any_finite) return false;

  // 1. greedy
  if (p.temperature < 1e-7f) {
    float best = -CUDART_INF_F;
    int64_t bi = INT64_MAX;
    for (int64_t i = tid; i < V; i += kThreads)
      if (s[i] > best) { best = s[i]; bi = i; }
    // block argmax: larger value wins, ties -> smaller index
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    __shared__ int64_t rbi[kWarps];
    const int w = tid >> 5, l = tid & 31;
    if (l == 0) { sh.rf[w] = best; rbi[w] = bi; }
    __syncthreads();
    best = sh.rf[l];
    bi = rbi[l];
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    const int64_t idx = (best == -CUDART_INF_F || bi == INT64_MAX) ? 0 : bi;  // sampling.rs:233-243
    // lightweight_logprob (sampling.rs:246-251)
    float mx = -CUDART_INF_F;
    for (int64_t i = tid; i < V; i += kThreads) mx = fmaxf(mx, s[i]);
    mx = block_max(mx, sh);
    double sd = 0.0;
    for (int64_t i = tid; i < V; i += kThreads) sd += (double)expf(s[i] - mx);
    const float se = (float)block_sum_d(sd, sh);
    token = idx;
    logprob = logf(__fdiv_rn(expf(s[idx] - mx), se));
    return true;
  }

  // 2. temperature
  if (p.temperature != 1.0f) {
    const float inv_t = __fdiv_rn(1.0f, p.temperature);
    for (int64_t i = tid; i < V; i += kThreads) s[i] = __fmul_rn(s[i], inv_t);
    __syncthreads();
  }
  // 3-5. penalties over the row's previous tokens: distinct ids with counts,
  // or dense per-token counts (a token with count 0 is untouched either way)
  const bool fp_on = p.presence_penalty != 0.f || p.frequency_penalty != 0.f;
  const bool rp_on = p.repetition_penalty != 1.0f;
  if (fp_on || rp_on) {
    auto penalise = [&](int64_t id, int c) {
      float v = s[id];
      if (fp_on) {
        v = __fsub_rn(v, __fmul_rn((float)c, p.frequency_penalty));
        if (p.presence_penalty != 0.f) v = __fsub_rn(v, p.presence_penalty);
      }
      if (rp_on)
        for (int t = 0; t < c; t++) v = v > 0.f ? __fdiv_rn(v, p.repetition_penalty) : __fmul_rn(v, p.repetition_penalty);
      s[id] = v;
    };
    if (a.dense_counts) {
      const int32_t* cnt = a.dense_counts + (int64_t)row * V;
      for (int64_t i = tid; i < V; i += kThreads) {
        const int c = cnt[i];
        if (c > 0) penalise(i, c);
      }
    } else if (a.pen_off) {
      for (int j = a.pen_off[row] + tid; j < a.pen_off[row + 1]; j += kThreads) {
        const int64_t id = a.pen_ids[j];
        if (id >= 0 && id < V) penalise(id, a.pen_cnt[j]);
      }
    }
    __syncthreads();
  }

  // 6. top-k: threshold = the k-th largest score
  if (p.top_k > 0 && (int64_t)p.top_k < V) {
    uint32_t prefix = 0, pmask = 0;
    u64 want = (u64)p.top_k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int d = tid; d < 256; d += kThreads) sh.cnt[d] = 0;
      __syncthreads();
      for (int64_t base = 0; base < V; base += kThreads) {
        const int64_t i = base + tid;
        uint32_t d = 0xffffffffu;
        if (i < V) {
          const uint32_t k = ord_key(s[i]);
          if ((k & pmask) == prefix) d = (k >> shift) & 255u;
        }
        hist_add(d, 0, sh, false);
      }
      __syncthreads();
      pick_digit(sh, want, false);
      // the k-th largest exists (k < V), so a digit is always found
      want -= sh.above;
      prefix |= sh.digit << shift;
      pmask |= 255u << shift;
      __syncthreads();
    }
    const float thr = key_value(prefix);
    for (int64_t i = tid; i < V; i += kThreads)
      if (s[i] < thr) s[i] = -CUDART_INF_F;
    __syncthreads();
  }

  // 7. top-p. Probabilities fall in the order of the scores (expf and the
  // division by the sum are monotone), so the descending-probability prefix is
  // found by a radix select over score keys, weighting each bucket by its
  // elements' probability mass; equal probabilities, which the reference leaves
  // to sort_unstable, are ordered by score, then by index.
  if (p.top_p > 0.f && p.top_p < 1.0f) {
    float mx = -CUDART_INF_F;
    for (int64_t i = tid; i < V; i += kThreads)
      if (finite_f(s[i])) mx = fmaxf(mx, s[i]);
    mx = block_max(mx, sh);
    const float se = softmax_sum(s, V, mx, sh);
    if (se > 0.f) {
      const u64 target = (u64)ceil((double)p.top_p * kFix);
      uint32_t prefix = 0, pmask = 0;
      u64 above = 0;  // mass of keys strictly above the current range
      bool keep_all = false;
      uint32_t ties = 0;  // elements with the cut's score
      for (int shift = 24; shift >= 0 && !keep_all; shift -= 8) {
        for (int d = tid; d < 256; d += kThreads) { sh.cnt[d] = 0; sh.mass[d] = 0; }
        __syncthreads();
        for (int64_t base = 0; base < V; base += kThreads) {
          const int64_t i = base + tid;
          uint32_t d = 0xffffffffu;
          u64 m = 0;
          if (i < V) {
            const float sv = s[i];
            const uint32_t k = ord_key(sv);
            if ((k & pmask) == prefix) {
              d = (k >> shift) & 255u;
              m = fix_of(prob_of(sv, mx, se));
            }
          }
          hist_add(d, m, sh, true);
        }
        __syncthreads();
        pick_digit(sh, target - above, true);
        if (!sh.found) {
          keep_all = true;  // the whole mass stays below top_p: nothing is cut
        } else {
          above += sh.above;
          prefix |= sh.digit << shift;
          pmask |= 255u << shift;
          if (shift == 0) ties = sh.cnt[sh.digit];
        }
        __syncthreads();
      }
      if (!keep_all) {
        const u64 mk = fix_of(prob_of(key_value(prefix), mx, se));
        const u64 need = target - above;
        const u64 j = mk ? (need + mk - 1) / mk : (u64)ties;  // tied elements the prefix needs
        if (j >= ties) {
          // the cut splits no tie: keep every score at or above the cut's
          for (int64_t i = tid; i < V; i += kThreads)
            if (ord_key(s[i]) < prefix) s[i] = -CUDART_INF_F;
          __syncthreads();
        } else {
          // ties at the cut keep the first j by index: contiguous chunks per thread
          const int64_t chunk = (V + kThreads - 1) / kThreads;
          const int64_t lo = tid * chunk, hi = min(V, lo + chunk);
          uint32_t mine = 0;
          for (int64_t i = lo; i < hi; i++) mine += ord_key(s[i]) == prefix;
          uint32_t incl = mine;
          for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
            if ((tid & 31) >= o) incl += t;
          }
          if ((tid & 31) == 31) sh.ri[tid >> 5] = (int)incl;
          __syncthreads();
          uint32_t rank = 0;
          for (int w = 0; w < (tid >> 5); w++) rank += (uint32_t)sh.ri[w];
          rank += incl - mine;
          for (int64_t i = lo; i < hi; i++) {
            const uint32_t k = ord_key(s[i]);
            bool keep = k > prefix;
            if (k == prefix) keep = (rank++ < j);
            if (!keep) s[i] = -CUDART_INF_F;
          }
          __syncthreads();
        }
      }
    }
  }

  // 8-9. softmax of what is left; nothing finite -> AllTokensMasked
  float mx = -CUDART_INF_F;
  for (int64_t i = tid; i < V; i += kThreads)
    if (finite_f(s[i])) mx = fmaxf(mx, s[i]);
  mx = block_max(mx, sh);
  if (mx == -CUDART_INF_F) return false;
  const float se = softmax_sum(s, V, mx, sh);
  if (!(se > 0.f) || !isfinite(se)) return false;

  // 10. multinomial: first i with R < prefix mass (index order), else the last token
  const float r = a.uniforms[row];
  // per-warp contiguous ranges, 32-element slices
  const int64_t span = ((V + kWarps - 1) / kWarps + 31) / 32 * 32;
  const int w = tid >> 5, l = tid & 31;
  u64 wsum = 0;
  for (int64_t i = w * span + l; i < min(V, (int64_t)(w + 1) * span); i += 32) wsum += fix_of(prob_of(s[i], mx, se));
  for (int o = 16; o; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  __syncthreads();
  if (l == 0) sh.ru[w] = wsum;
  __syncthreads();
  if (w == 0) {
    // r < cdf(i) in exact arithmetic  <=>  floor(r * 2^40) < prefix mass(i)
    const u64 R = (u64)floor((double)r * kFix);
    u64 acc = 0;
    int ww = -1;
    for (int k = 0; k < kWarps; k++) {
      if (acc + sh.ru[k] > R) { ww = k; break; }
      acc += sh.ru[k];
    }
    if (l == 0) { sh.found = ww; sh.above = acc; sh.draw = R; }
  }
  __syncthreads();
  const int ww = sh.found;
  int64_t tok = V - 1;  // sampling.rs:286-289: the rounding guard returns the last token
  if (ww >= 0) {
    if (w == ww) {
      const u64 R = sh.draw;
      u64 acc = sh.above;
      const int64_t end = min(V, (int64_t)(ww + 1) * span);
      for (int64_t base = (int64_t)ww * span; base < end; base += 32) {
        const int64_t i = base + l;
        const u64 m = i < end ? fix_of(prob_of(s[i], mx, se)) : 0;
        u64 incl = m;
        for (int o = 1; o < 32; o <<= 1) {
          const u64 t = __shfl_up_sync(0xffffffffu, incl, o);
          if (l >= o) incl += t;
        }
        const unsigned hit = __ballot_sync(0xffffffffu, i < end && acc + incl > R);
        if (hit) {
          if (l == 0) sh.token = base + __ffs(hit) - 1;
          break;
        }
        acc += __shfl_sync(0xffffffffu, incl, 31);
      }
    }
    __syncthreads();
    tok = sh.token;
  }
  token = tok;
  logprob = logf(prob_of(s[tok], mx, se));
  return true;
}

__global__ void __launch_bounds__(kThreads, 1) sample_kernel(SampleArgs a, int use_smem) {
  extern __shared__ float dyn[];
  __shared__ Shared sh;
  const int row = blockIdx.x;
  float* s = use_smem ? dyn : a.scratch + (int64_t)row * a.vocab;
  const float* lg = a.logits + (int64_t)row * a.vocab;
  const zl_sampling_params p = a.params[row];
  bool masked = a.allowed && (!a.mask_rows || a.mask_rows[row]);
  int status = 0;
  int64_t token = 0;
  float logprob = -CUDART_INF_F;
  bool ok = sample_row(a, p, row, s, lg, masked, sh, token, logprob);
  if (!ok && masked && a.fallback_unmasked) {
    __syncthreads();
    status |= ZL_SAMPLE_FELL_BACK;
    ok = sample_row(a, p, row, s, lg, false, sh, token, logprob);
  }
  if (!ok) {
    status |= ZL_SAMPLE_ALL_MASKED;
    token = 0;  // engine.rs:214-217 keeps going with token 0
    logprob = -CUDART_INF_F;
  }
  if (threadIdx.x == 0) {
    a.token_ids[row] = token;
    // the engine appends whatever token it got to output_tokens (engine.rs:219-222)
    if (a.dense_counts && a.update_counts) a.dense_counts[(int64_t)row * a.vocab + token] += 1;
    a.logprobs[row] = logprob;
    if (a.row_status) a.row_status[row] = status;
  }
}

}  // namespace

using namespace zl;

extern "C" zl_status zl_sample(zl_ctx* ctx, const float* logits, int num_rows, int64_t vocab,
                               const zl_sampling_params* params, const uint32_t* allowed_bits,
                               const uint8_t* mask_rows, int64_t mask_len, const int32_t* penalty_offsets,
                               const int64_t* penalty_ids, const int32_t* penalty_counts,
                               int32_t* dense_counts, int update_dense_counts, const float* uniforms,
                               int fallback_unmasked, int64_t* token_ids, float* logprobs, int32_t* row_status,
                               zl_stream stream) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  if (num_rows < 0) return set_error(ZL_ERR_INVALID_ARG, "sample: num_rows < 0");
  if (num_rows == 0) return ZL_OK;
  if (vocab <= 0) return set_error(ZL_ERR_INVALID_ARG, "sample: empty logits (SamplingError::EmptyLogits)");
  if (vocab >= (int64_t)1 << 31) return set_error(ZL_ERR_INVALID_ARG, "sample: vocab too large");
  if (!logits || !params || !uniforms || !token_ids || !logprobs)
    return set_error(ZL_ERR_INVALID_ARG, "sample: null argument");
  if (allowed_bits && mask_len < 0) return set_error(ZL_ERR_INVALID_ARG, "sample: mask_len < 0");
  if (penalty_offsets && (!penalty_ids || !penalty_counts))
    return set_error(ZL_ERR_INVALID_ARG, "sample: penalty ids/counts missing");
  if (penalty_offsets && dense_counts)
    return set_error(ZL_ERR_INVALID_ARG, "sample: give penalty lists or dense counts, not both");
  SampleArgs a{};
  a.logits = logits;
  a.vocab = vocab;
  a.params = params;
  a.allowed = allowed_bits;
  a.mask_rows = mask_rows;
  a.mask_len = allowed_bits ? mask_len : 0;
  a.mask_words = (a.mask_len + 31) / 32;
  a.pen_off = penalty_offsets;
  a.pen_ids = penalty_ids;
  a.pen_cnt = penalty_counts;
  a.dense_counts = dense_counts;
  a.update_counts = update_dense_counts;
  a.uniforms = uniforms;
  a.fallback_unmasked = fallback_unmasked;
  a.token_ids = token_ids;
  a.logprobs = logprobs;
  a.row_status = row_status;
  const int use_smem = vocab <= kMaxSmemVocab;
  size_t smem = 0;
  if (use_smem) {
    smem = (size_t)vocab * 4;
    static unsigned attr_set = 0;
    if (!(attr_set & (1u << (ctx->device & 31)))) {
      ZL_CUDA_TRY(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kMaxSmemVocab * 4));
      attr_set |= 1u << (ctx->device & 31);
    }
  } else {
    const size_t need = (size_t)num_rows * vocab * 4;
    if (ctx->sample_scratch_bytes < need) {
      if (ctx->sample_scratch) {
        ZL_CUDA_TRY(cudaDeviceSynchronize());
        ZL_CUDA_TRY(cudaFree(ctx->sample_scratch));
        ctx->sample_scratch = nullptr;
        ctx->sample_scratch_bytes = 0;
      }
      ZL_CUDA_TRY(cudaMalloc(&ctx->sample_scratch, need));
      ctx->sample_scratch_bytes = need;
    }
    a.scratch = reinterpret_cast<float*>(ctx->sample_scratch);
  }
  sample_kernel<<<num_rows, kThreads, smem, S(stream)>>>(a, use_smem);
  ZL_LAUNCH_CHECK(ctx);
  return ZL_OK;
}
