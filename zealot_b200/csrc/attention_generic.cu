// attention_generic.cu -- CUDA-core attention for every shape the tensor-core
// kernels do not cover (fp32 pools, head_dim != 128, odd block sizes, wide
// GQA groups), plus the partial-triple merge.
//
// One CTA of 128 threads owns one (query row, head). Keys are consumed in
// chunks of 128: each thread scores one key (serial fp32 dot over d, as the
// reference CpuAttention does, src/attention/mod.rs:66-71), the CTA reduces
// the chunk max and sum, and the threads that own output dims accumulate
// p*v with an online rescale. fp32 accumulation throughout.
#include "zl_internal.h"

#include <cfloat>

namespace {

constexpr int kThreads = 128;
constexpr int kMaxDim = 256;

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  return r;
}
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = (red[0] + red[1]) + (red[2] + red[3]);
  __syncthreads();
  return r;
}

struct AttendShared {
  float q[kMaxDim];
  float p[kThreads];
  int64_t row[kThreads];
  float red[4];
  int first_neg;
};

// Online-softmax attention of one query (already in sh.q) over keys
// [j0, j1). row_of(j) returns the element offset of key j's row in the K/V
// arrays, or -1 for a masked key. Results: m (natural-log units), l, acc[].
template <typename T, typename RowOf>
__device__ void attend(const T* __restrict__ kbase, const T* __restrict__ vbase, int d, float scale,
                       int64_t j0, int64_t j1, RowOf row_of, AttendShared& sh, float& m_out,
                       float& l_out, float acc[2]) {
  const int tid = threadIdx.x;
  float m = -INFINITY, l = 0.f;
  acc[0] = acc[1] = 0.f;
  for (int64_t base = j0; base < j1; base += kThreads) {
    const int64_t j = base + tid;
    float s = -INFINITY;
    int64_t row = -1;
    if (j < j1) {
      row = row_of(j);
      if (row >= 0) {
        const T* kr = kbase + row;
        float dot = 0.f;
        for (int e = 0; e < d; e++) dot = __fadd_rn(dot, __fmul_rn(sh.q[e], to_f(kr[e])));
        s = __fmul_rn(dot, scale);
      }
    }
    const float cmax = block_max(s, sh.red);
    const float m_new = fmaxf(m, cmax);
    float p = 0.f;
    if (row >= 0 && m_new != -INFINITY) p = expf(s - m_new);
    const float alpha = (m == -INFINITY) ? 0.f : expf(m - m_new);
    sh.p[tid] = p;
    sh.row[tid] = row;
    const float psum = block_sum(p, sh.red);  // has a barrier: p/row visible
    l = l * alpha + psum;
    const int64_t rem = j1 - base;
    const int cnt = rem < kThreads ? (int)rem : kThreads;
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const int e = tid + r * kThreads;
      if (e < d) {
        float a = acc[r] * alpha;
        for (int jj = 0; jj < cnt; jj++) {
          const float pj = sh.p[jj];
          if (pj != 0.f) a = fmaf(pj, to_f(vbase[sh.row[jj] + e]), a);
        }
        acc[r] = a;
      }
    }
    if (m_new != -INFINITY) m = m_new;
    __syncthreads();
  }
  m_out = m;
  l_out = l;
}

// ------------------------------------------------------------------ decode

template <typename T>
__global__ void __launch_bounds__(kThreads)
decode_generic_kernel(const T* __restrict__ q, const T* __restrict__ k_pool,
                      const T* __restrict__ v_pool, const int32_t* __restrict__ block_tables,
                      const int32_t* __restrict__ seq_lens, const int32_t* __restrict__ tok_begin,
                      T* __restrict__ out, float* __restrict__ m_out, float* __restrict__ l_out,
                      float* __restrict__ o_out, int H, int Hkv, int d, int bs, int max_blocks,
                      int64_t num_blocks, float scale, int gqa_modulo, int* status) {
  __shared__ AttendShared sh;
  const int b = blockIdx.x / H;
  const int h = blockIdx.x - b * H;
  const int tid = threadIdx.x;
  const int kvh = gqa_modulo ? h % Hkv : h / (H / Hkv);
  const int64_t qoff = ((int64_t)b * H + h) * d;
  for (int e = tid; e < d; e += kThreads) sh.q[e] = to_f(q[qoff + e]);
  int64_t len = max(seq_lens[b], 0);
  int64_t nblk = (len + bs - 1) / bs;
  if (nblk > max_blocks) {
    if (tid == 0) atomicOr(status, ZL_DEV_OOB);
    nblk = max_blocks;
    len = nblk * bs;
  }
  // A negative table entry ends the sequence (paged_attention.cu:66-67).
  if (tid == 0) sh.first_neg = (int)nblk;
  __syncthreads();
  const int32_t* table = block_tables + (int64_t)b * max_blocks;
  for (int64_t t = tid; t < nblk; t += kThreads)
    if (table[t] < 0) atomicMin(&sh.first_neg, (int)t);
  __syncthreads();
  const int64_t n_end = min(len, (int64_t)sh.first_neg * bs);
  const int64_t j0 = tok_begin ? max(tok_begin[b], 0) : 0;
  auto row_of = [&](int64_t j) -> int64_t {
    const int64_t blk = table[j / bs];
    if (blk >= num_blocks) {
      atomicOr(status, ZL_DEV_OOB);
      return -1;
    }
    return ((blk * Hkv + kvh) * bs + (j % bs)) * d;
  };
  float m, l, acc[2];
  attend<T>(k_pool, v_pool, d, scale, j0, n_end, row_of, sh, m, l, acc);
  if (o_out) {  // partial triple
    if (tid == 0) {
      m_out[(int64_t)b * H + h] = m;
      l_out[(int64_t)b * H + h] = l;
    }
    for (int r = 0; r < 2; r++) {
      const int e = tid + r * kThreads;
      if (e < d) o_out[qoff + e] = acc[r];
    }
  } else {
    const float inv = l > 0.f ? 1.f / l : 0.f;
    for (int r = 0; r < 2; r++) {
      const int e = tid + r * kThreads;
      if (e < d) out[qoff + e] = from_f<T>(acc[r] * inv);
    }
  }
}

// ----------------------------------------------------------------- prefill

template <typename T>
__global__ void __launch_bounds__(kThreads)
prefill_generic_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                       const int32_t* __restrict__ cu_seqlens, T* __restrict__ out, int H, int Hkv,
                       int d, float scale, int causal, int gqa_modulo, int64_t total_tokens,
                       int* status) {
  __shared__ AttendShared sh;
  // grid: x = row within the sequence, y = head, z = sequence
  const int64_t i = blockIdx.x;
  const int h = blockIdx.y;
  const int64_t start = cu_seqlens[blockIdx.z], end = cu_seqlens[blockIdx.z + 1];
  // A sequence outside [0, total_tokens], running backwards, or longer than the
  // launch's rows (gridDim.x = max_seq_len) is reported and skipped: no access
  // leaves the caller's buffers.
  if (start < 0 || end < start || end > total_tokens || end - start > (int64_t)gridDim.x) {
    if (threadIdx.x == 0 && i == 0) atomicOr(status, ZL_DEV_OOB);
    return;
  }
  if (start + i >= end) return;
  const int tid = threadIdx.x;
  const int64_t row = start + i;
  const int kvh = gqa_modulo ? h % Hkv : h / (H / Hkv);
  const int64_t qoff = (row * H + h) * d;
  for (int e = tid; e < d; e += kThreads) sh.q[e] = to_f(q[qoff + e]);
  __syncthreads();
  const int64_t n = causal ? i + 1 : end - start;
  auto row_of = [&](int64_t j) -> int64_t { return ((start + j) * Hkv + kvh) * d; };
  float m, l, acc[2];
  attend<T>(k, v, d, scale, 0, n, row_of, sh, m, l, acc);
  const float inv = l > 0.f ? 1.f / l : 0.f;
  for (int r = 0; r < 2; r++) {
    const int e = tid + r * kThreads;
    if (e < d) out[qoff + e] = from_f<T>(acc[r] * inv);
  }
}

// ------------------------------------------------------------------- merge

template <typename T>
__global__ void __launch_bounds__(256)
merge_kernel(const float* __restrict__ m, const float* __restrict__ l, const float* __restrict__ o,
             int P, int64_t rows, int d, T* __restrict__ out) {
  const int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float M = -INFINITY;
  for (int p = 0; p < P; p++) M = fmaxf(M, m[(int64_t)p * rows + r]);
  float wsum = 0.f;
  for (int p = 0; p < P; p++) {
    const float mp = m[(int64_t)p * rows + r];
    if (mp != -INFINITY) wsum += expf(mp - M) * l[(int64_t)p * rows + r];
  }
  const float inv = (M == -INFINITY || wsum == 0.f) ? 0.f : 1.f / wsum;
  for (int e = lane; e < d; e += 32) {
    float acc = 0.f;
    for (int p = 0; p < P; p++) {
      const float mp = m[(int64_t)p * rows + r];
      if (mp != -INFINITY) acc = fmaf(expf(mp - M), o[((int64_t)p * rows + r) * d + e], acc);
    }
    out[r * d + e] = from_f<T>(acc * inv);
  }
}

}  // namespace

namespace zl {

zl_status launch_decode_generic(zl_ctx* ctx, const void* q, const void* k_pool, const void* v_pool,
                                const int32_t* block_tables, const int32_t* seq_lens,
                                const int32_t* tok_begin, void* out, float* m_out, float* l_out,
                                float* o_out, int B, int H, int Hkv, int d, int bs, int max_blocks,
                                int64_t num_blocks, float scale, zl_gqa_map map, zl_dtype dtype,
                                cudaStream_t st) {
  if (d > kMaxDim)
    return set_error(ZL_ERR_UNSUPPORTED, "paged decode: head_dim %d > %d", d, kMaxDim);
  const int64_t grid = (int64_t)B * H;
  if (grid == 0) return ZL_OK;
  if (grid > 0x7fffffff) return set_error(ZL_ERR_INVALID_ARG, "paged decode: B*H too large");
  const int mod = map == ZL_GQA_MODULO;
  if (dtype == ZL_F32)
    decode_generic_kernel<float><<<(unsigned)grid, kThreads, 0, st>>>(
        (const float*)q, (const float*)k_pool, (const float*)v_pool, block_tables, seq_lens,
        tok_begin, (float*)out, m_out, l_out, o_out, H, Hkv, d, bs, max_blocks, num_blocks, scale,
        mod, ctx->d_status);
  else
    decode_generic_kernel<__nv_bfloat16><<<(unsigned)grid, kThreads, 0, st>>>(
        (const __nv_bfloat16*)q, (const __nv_bfloat16*)k_pool, (const __nv_bfloat16*)v_pool,
        block_tables, seq_lens, tok_begin, (__nv_bfloat16*)out, m_out, l_out, o_out, H, Hkv, d, bs,
        max_blocks, num_blocks, scale, mod, ctx->d_status);
  ZL_LAUNCH_CHECK(ctx);
  return ZL_OK;
}

zl_status launch_prefill_generic(zl_ctx* ctx, const void* q, const void* k, const void* v,
                                 const int32_t* cu_seqlens, int num_seqs, int max_seq_len,
                                 int64_t total_tokens, void* out, int H, int Hkv, int d, float scale,
                                 int causal, zl_gqa_map map, zl_dtype dtype, cudaStream_t st) {
  if (d > kMaxDim) return set_error(ZL_ERR_UNSUPPORTED, "prefill: head_dim %d > %d", d, kMaxDim);
  if (num_seqs == 0 || max_seq_len == 0 || H == 0) return ZL_OK;
  if (num_seqs > 65535 || H > 65535)
    return set_error(ZL_ERR_INVALID_ARG, "prefill: more than 65535 sequences or heads");
  dim3 grid((unsigned)max_seq_len, (unsigned)H, (unsigned)num_seqs);
  const int mod = map == ZL_GQA_MODULO;
  if (dtype == ZL_F32)
    prefill_generic_kernel<float><<<grid, kThreads, 0, st>>>(
        (const float*)q, (const float*)k, (const float*)v, cu_seqlens, (float*)out, H, Hkv, d,
        scale, causal, mod, total_tokens, ctx->d_status);
  else
    prefill_generic_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(
        (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, cu_seqlens,
        (__nv_bfloat16*)out, H, Hkv, d, scale, causal, mod, total_tokens, ctx->d_status);
  ZL_LAUNCH_CHECK(ctx);
  return ZL_OK;
}

zl_status launch_merge(zl_ctx* ctx, const float* m, const float* l, const float* o, int P,
                       int64_t rows, int d, void* out, zl_dtype dtype, cudaStream_t st) {
  if (rows == 0) return ZL_OK;
  const int warps = 8;
  const int64_t blocks = (rows + warps - 1) / warps;
  if (dtype == ZL_F32)
    merge_kernel<float><<<(unsigned)blocks, warps * 32, 0, st>>>(m, l, o, P, rows, d, (float*)out);
  else
    merge_kernel<__nv_bfloat16><<<(unsigned)blocks, warps * 32, 0, st>>>(m, l, o, P, rows, d,
                                                                           (__nv_bfloat16*)out);
  ZL_LAUNCH_CHECK(ctx);
  return ZL_OK;
}

}  // namespace zl
