// decoder.cu -- one continuous-batching engine step of a decoder model on the
// GPU: the layer loop of the reference CUDA runner (src/cuda_runner.rs:303-607)
// batched over every sequence of the step instead of one sequence at a time.
//
// Per layer:  h = rmsnorm(x) ; q,k,v = h W^T ; reshape_and_cache(k, v)
//             o[prefill rows] = varlen causal prefill ; o[decode rows] = paged decode
//             x += o Wo^T ; h = rmsnorm(x) ; g,u = h Wgu^T ; x += (silu(g) * u) Wd^T
// then        logits = rmsnorm(x[last rows]) lm_head^T            (fp32 out)
//
// The GEMMs are plain bf16 library GEMMs (cuBLAS, fp32 accumulate, opened with
// dlopen so the library has no link-time cuBLAS dependency); the residual adds
// ride on the GEMM (beta = 1 into the residual stream). Steps of 512 rows or
// more compute gate/up and SiLU-gate in one tcgen05 kernel of this library
// (gemm_swiglu.cu); smaller steps use the library GEMM and a small kernel.
// RMSNorm and the embedding gather are small kernels; attention uses this
// library's kernels. As in the reference runner there is no rotary embedding.
#include <dlfcn.h>

#include <mutex>

#include "zl_internal.h"

namespace {

// ------------------------------------------------------------------- cuBLAS
typedef int cublasStatus_t;
typedef void* cublasHandle_t;
enum { CUBLAS_OP_N = 0, CUBLAS_OP_T = 1 };
enum { CUBLAS_COMPUTE_32F = 68 };
enum { CUBLAS_GEMM_DEFAULT = -1 };
enum { CUDA_R_32F_ = 0, CUDA_R_16BF_ = 14 };

struct CublasApi {
  cublasStatus_t (*Create)(cublasHandle_t*) = nullptr;
  cublasStatus_t (*Destroy)(cublasHandle_t) = nullptr;
  cublasStatus_t (*SetStream)(cublasHandle_t, cudaStream_t) = nullptr;
  cublasStatus_t (*GemmEx)(cublasHandle_t, int, int, int, int, int, const void*, const void*, int, int,
                           const void*, int, int, const void*, void*, int, int, int, int) = nullptr;
  cublasStatus_t (*SetWorkspace)(cublasHandle_t, void*, size_t) = nullptr;
  bool ok = false;
};

CublasApi& cublas() {
  static CublasApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libcublas.so.12", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    a.Create = (decltype(a.Create))dlsym(h, "cublasCreate_v2");
    a.Destroy = (decltype(a.Destroy))dlsym(h, "cublasDestroy_v2");
    a.SetStream = (decltype(a.SetStream))dlsym(h, "cublasSetStream_v2");
    a.GemmEx = (decltype(a.GemmEx))dlsym(h, "cublasGemmEx");
    a.SetWorkspace = (decltype(a.SetWorkspace))dlsym(h, "cublasSetWorkspace_v2");
    a.ok = a.Create && a.Destroy && a.SetStream && a.GemmEx && a.SetWorkspace;
  });
  return a;
}

// One cuBLAS handle per device, created on first use, with a workspace of its
// own so that no GEMM allocates (a step can then be captured in a CUDA graph).
constexpr size_t kCublasWorkspace = 32u << 20;
cublasHandle_t cublas_handle(int dev) {
  static cublasHandle_t handles[64] = {};
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!handles[dev] && cublas().ok) {
    void* ws = nullptr;
    if (cudaMalloc(&ws, kCublasWorkspace) != cudaSuccess) return nullptr;
    cublasHandle_t h = nullptr;
    if (cublas().Create(&h) != 0) { cudaFree(ws); return nullptr; }
    if (cublas().SetWorkspace(h, ws, kCublasWorkspace) != 0) {
      cublas().Destroy(h);
      cudaFree(ws);
      return nullptr;
    }
    handles[dev] = h;  // handle and workspace live until the process exits
  }
  return handles[dev];
}

// Row-major Y[M][N] (+)= X[M][K] W[N][K]^T  (torch Linear layout), bf16 in,
// fp32 accumulate, Y bf16 (or fp32 when y_f32).
zl_status linear(cublasHandle_t h, cudaStream_t st, const void* x, const void* w, void* y, int64_t M,
                 int64_t N, int64_t K, bool accumulate, bool y_f32 = false) {
  if (M == 0) return ZL_OK;
  const float alpha = 1.f, beta = accumulate ? 1.f : 0.f;
  CublasApi& c = cublas();
  if (c.SetStream(h, st) != 0) return zl::set_error(ZL_ERR_CUDA, "cublasSetStream failed");
  // column-major view: Y^T[N][M] = W[N][K] * X^T[K][M]
  const cublasStatus_t r =
      c.GemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, (int)N, (int)M, (int)K, &alpha, w, CUDA_R_16BF_, (int)K, x,
               CUDA_R_16BF_, (int)K, &beta, y, y_f32 ? CUDA_R_32F_ : CUDA_R_16BF_, (int)N,
               CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
  if (r != 0) return zl::set_error(ZL_ERR_CUDA, "cublasGemmEx failed (%d) for %lldx%lldx%lld", r,
                                   (long long)M, (long long)N, (long long)K);
  return ZL_OK;
}

// ------------------------------------------------------------------ kernels
__global__ void embed_bf16_kernel(const int64_t* __restrict__ ids, int64_t T, const __nv_bfloat16* __restrict__ table,
                                  int64_t vocab, int hidden, __nv_bfloat16* __restrict__ out) {
  const int64_t chunks = hidden / 8;  // 16-byte chunks
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < T * chunks;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / chunks, c = i - t * chunks;
    const int64_t id = ids[t];
    uint4 v = make_uint4(0, 0, 0, 0);
    if (id >= 0 && id < vocab) v = reinterpret_cast<const uint4*>(table + id * hidden)[c];
    reinterpret_cast<uint4*>(out + t * hidden)[c] = v;
  }
}

// out[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * w ; one CTA per row (src/attention/
// kernels/rms_norm.cu:4-55 computes the same with a scalar loop per row).
__global__ void __launch_bounds__(256)
rmsnorm_bf16_kernel(const __nv_bfloat16* __restrict__ x, const int32_t* __restrict__ rows,
                    const __nv_bfloat16* __restrict__ w, int hidden, float eps, __nv_bfloat16* __restrict__ out) {
  const int64_t r = rows ? rows[blockIdx.x] : blockIdx.x;
  const __nv_bfloat16* xr = x + r * hidden;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < hidden; i += blockDim.x * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + i);
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float2 f = __bfloat1622float2(p[k]);
      ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
    }
  }
  __shared__ float red[8];
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int k = 0; k < (int)(blockDim.x >> 5); k++) tot += red[k];
  const float inv = rsqrtf(tot / hidden + eps);
  __nv_bfloat16* orow = out + (int64_t)blockIdx.x * hidden;
  for (int i = threadIdx.x * 8; i < hidden; i += blockDim.x * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + i);
    const uint4 g = *reinterpret_cast<const uint4*>(w + i);
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
    const __nv_bfloat162* q = reinterpret_cast<const __nv_bfloat162*>(&g);
    uint4 o;
    __nv_bfloat162* po = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float2 f = __bfloat1622float2(p[k]), gw = __bfloat1622float2(q[k]);
      po[k] = __floats2bfloat162_rn(f.x * inv * gw.x, f.y * inv * gw.y);
    }
    *reinterpret_cast<uint4*>(orow + i) = o;
  }
}

// act[t][i] = silu(gu[t][i]) * gu[t][I + i]  (gate then up, as activation.cu:4-12)
__global__ void silu_mul_bf16_kernel(const __nv_bfloat16* __restrict__ gu, int64_t T, int inter,
                                     __nv_bfloat16* __restrict__ act) {
  const int64_t chunks = inter / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < T * chunks;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / chunks, c = i - t * chunks;
    const uint4 g = reinterpret_cast<const uint4*>(gu + t * 2 * inter)[c];
    const uint4 u = reinterpret_cast<const uint4*>(gu + t * 2 * inter + inter)[c];
    const __nv_bfloat162* pg = reinterpret_cast<const __nv_bfloat162*>(&g);
    const __nv_bfloat162* pu = reinterpret_cast<const __nv_bfloat162*>(&u);
    uint4 o;
    __nv_bfloat162* po = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float2 a = __bfloat1622float2(pg[k]), b = __bfloat1622float2(pu[k]);
      po[k] = __floats2bfloat162_rn(a.x / (1.f + expf(-a.x)) * b.x, a.y / (1.f + expf(-a.y)) * b.y);
    }
    reinterpret_cast<uint4*>(act + t * inter)[c] = o;
  }
}

// y[t] = [q | k | v] rows of one fused projection -> q[t][nq], k[t][nk], v[t][nk]
// (16-byte chunks; nq, nk multiples of 8).
__global__ void split_qkv_bf16_kernel(const __nv_bfloat16* __restrict__ y, int64_t T, int nq, int nk,
                                      __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k,
                                      __nv_bfloat16* __restrict__ v) {
  const int64_t row = (nq + 2 * nk) / 8;  // chunks per fused row
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < T * row;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / row;
    const int c = (int)(i - t * row);
    const uint4 val = reinterpret_cast<const uint4*>(y)[i];
    if (c < nq / 8) reinterpret_cast<uint4*>(q + t * nq)[c] = val;
    else if (c < (nq + nk) / 8) reinterpret_cast<uint4*>(k + t * nk)[c - nq / 8] = val;
    else reinterpret_cast<uint4*>(v + t * nk)[c - (nq + nk) / 8] = val;
  }
}

// Steps with at most this many rows read wq, wk and wv with one GEMM when they are
// stored back to back: a few rows make the projections weight-read-bound, and
// the 1024-wide k and v products alone reach only a small part of HBM
// bandwidth. The fused product goes to the gate/up buffer (free at that point
// of the layer) and a copy kernel splits it.
constexpr int64_t kFusedQkvRows = 256;

// Steps with at least this many rows run the gate/up projection and SiLU-gate
// as one tcgen05 kernel (zl_linear_swiglu). Measured on one B200 against the
// library GEMM + elementwise kernel at hidden 4096 / intermediate 14336:
// 0.707 vs 0.981 ms at 4,344 rows, 0.187 vs 0.256 ms at 1,024; at 248 and 32
// rows (only 112 of the 148 SMs get an output strip) 0.086 vs 0.081 and 0.067
// vs 0.055 ms, so decode-sized steps keep the two-kernel form.
constexpr int64_t kFusedMlpRows = 512;

unsigned grid_of(int64_t work, int num_sms) {
  int64_t g = (work + 255) / 256;
  const int64_t cap = (int64_t)num_sms * 16;
  return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace

using namespace zl;

extern "C" zl_status zl_decoder_step(zl_ctx* ctx, const zl_decoder* m, void* const* k_pools,
                                     void* const* v_pools, int64_t num_blocks, int block_size,
                                     const zl_step_batch* b, float* logits, zl_stream stream) {
  zl_status s = bind_device(ctx);
  if (s != ZL_OK) return s;
  if (!m || !k_pools || !v_pools || !b || !logits)
    return set_error(ZL_ERR_INVALID_ARG, "decoder_step: null argument");
  const int hid = m->hidden, H = m->num_heads, Hkv = m->num_kv_heads, d = m->head_dim, I = m->intermediate;
  if (hid <= 0 || hid % 8 || I <= 0 || I % 8 || H <= 0 || Hkv <= 0 || H % Hkv || d <= 0 || m->num_layers <= 0 ||
      m->vocab <= 0 || !m->layers || !m->embed || !m->final_norm || !m->lm_head)
    return set_error(ZL_ERR_INVALID_ARG, "decoder_step: bad model description");
  const int64_t P = b->prefill_tokens, D = b->num_decode, T = P + D;
  if (P < 0 || D < 0 || b->num_prefill < 0 || b->num_last < 0 || (P > 0 && !b->cu_prefill) ||
      (D > 0 && (!b->block_tables || !b->seq_lens)) || !b->tokens || !b->slot_mapping || !b->last_rows)
    return set_error(ZL_ERR_INVALID_ARG, "decoder_step: bad batch description");
  if (T == 0) return ZL_OK;
  if (!cublas().ok) return set_error(ZL_ERR_CUDA, "libcublas.so.12 could not be loaded");
  cublasHandle_t hb = cublas_handle(ctx->device);
  if (!hb) return set_error(ZL_ERR_CUDA, "cublasCreate failed");
  cudaStream_t st = S(stream);

  // activations live in the context workspace
  // every buffer starts on a 256-byte boundary (vector loads, TMA bases)
  auto up = [](size_t n) { return (n + 255) & ~(size_t)255; };
  const size_t e = 2;
  const size_t off_x = 0, off_h = off_x + up(T * hid * e), off_q = off_h + up(T * hid * e),
               off_k = off_q + up(T * H * d * e), off_v = off_k + up(T * Hkv * d * e),
               off_o = off_v + up(T * Hkv * d * e), off_gu = off_o + up(T * H * d * e),
               off_a = off_gu + up(T * 2 * I * e), off_last = off_a + up(T * I * e),
               total = off_last + up((size_t)b->num_last * hid * e);
  // the split-KV workspace is separate: attention calls below may grow it
  if (ctx->activation_bytes < total) {
    if (ctx->activations) {
      ZL_CUDA_TRY(cudaStreamSynchronize(st));
      ZL_CUDA_TRY(cudaFree(ctx->activations));
      ctx->activations = nullptr;
      ctx->activation_bytes = 0;
    }
    ZL_CUDA_TRY(cudaMalloc(&ctx->activations, total));
    ctx->activation_bytes = total;
  }
  uint8_t* w = reinterpret_cast<uint8_t*>(ctx->activations);
  auto* x = reinterpret_cast<__nv_bfloat16*>(w + off_x);
  auto* h = reinterpret_cast<__nv_bfloat16*>(w + off_h);
  auto* q = reinterpret_cast<__nv_bfloat16*>(w + off_q);
  auto* k = reinterpret_cast<__nv_bfloat16*>(w + off_k);
  auto* v = reinterpret_cast<__nv_bfloat16*>(w + off_v);
  auto* o = reinterpret_cast<__nv_bfloat16*>(w + off_o);
  auto* gu = reinterpret_cast<__nv_bfloat16*>(w + off_gu);
  auto* a = reinterpret_cast<__nv_bfloat16*>(w + off_a);
  auto* last = reinterpret_cast<__nv_bfloat16*>(w + off_last);

  embed_bf16_kernel<<<grid_of(T * hid / 8, ctx->num_sms), 256, 0, st>>>(
      b->tokens, T, (const __nv_bfloat16*)m->embed, m->vocab, hid, x);
  ZL_LAUNCH_CHECK(ctx);
  for (int l = 0; l < m->num_layers; l++) {
    const zl_layer_weights& L = m->layers[l];
    rmsnorm_bf16_kernel<<<(unsigned)T, 256, 0, st>>>(x, nullptr, (const __nv_bfloat16*)L.attn_norm, hid,
                                                      m->rms_eps, h);
    ZL_LAUNCH_CHECK(ctx);
    const int64_t nq = (int64_t)H * d, nk = (int64_t)Hkv * d;
    const bool fused = T <= kFusedQkvRows && d % 8 == 0 && 2 * (int64_t)I >= nq + 2 * nk &&
                       (const uint8_t*)L.wk == (const uint8_t*)L.wq + nq * hid * e &&
                       (const uint8_t*)L.wv == (const uint8_t*)L.wk + nk * hid * e;
    if (fused) {
      if ((s = linear(hb, st, h, L.wq, gu, T, nq + 2 * nk, hid, false))) return s;
      split_qkv_bf16_kernel<<<grid_of(T * (nq + 2 * nk) / 8, ctx->num_sms), 256, 0, st>>>(
          gu, T, (int)nq, (int)nk, q, k, v);
      ZL_LAUNCH_CHECK(ctx);
    } else if ((s = linear(hb, st, h, L.wq, q, T, nq, hid, false)) ||
               (s = linear(hb, st, h, L.wk, k, T, nk, hid, false)) ||
               (s = linear(hb, st, h, L.wv, v, T, nk, hid, false))) {
      return s;
    }
    if ((s = zl_reshape_and_cache(ctx, k, v, k_pools[l], v_pools[l], b->slot_mapping, T, Hkv, d, block_size,
                                  num_blocks, ZL_BF16, stream)))
      return s;
    if (P > 0 && (s = zl_prefill_varlen(ctx, q, k, v, b->cu_prefill, b->num_prefill, b->max_prefill_len, P, o,
                                        H, Hkv, d, 0.f, 1, ZL_GQA_GROUPED, ZL_BF16, stream)))
      return s;
    if (D > 0 && (s = zl_paged_decode(ctx, q + P * H * d, k_pools[l], v_pools[l], b->block_tables, b->seq_lens,
                                      o + P * H * d, (int)D, H, Hkv, d, block_size, b->max_blocks_per_seq,
                                      num_blocks, 0.f, ZL_GQA_GROUPED, 0, ZL_BF16, stream)))
      return s;
    if ((s = linear(hb, st, o, L.wo, x, T, hid, (int64_t)H * d, true))) return s;
    rmsnorm_bf16_kernel<<<(unsigned)T, 256, 0, st>>>(x, nullptr, (const __nv_bfloat16*)L.mlp_norm, hid,
                                                      m->rms_eps, h);
    ZL_LAUNCH_CHECK(ctx);
    // gate/up + SiLU-gate: one kernel with the activation in its epilogue
    // (gemm_swiglu.cu) for steps of kFusedMlpRows rows or more; smaller steps
    // keep the library GEMM and the elementwise kernel (faster there).
    const zl_status f = T >= kFusedMlpRows ? launch_gemm_swiglu(ctx, h, L.w_gate_up, a, T, hid, I, st)
                                           : ZL_ERR_UNSUPPORTED;
    if (f == ZL_ERR_UNSUPPORTED) {
      if ((s = linear(hb, st, h, L.w_gate_up, gu, T, 2 * (int64_t)I, hid, false))) return s;
      silu_mul_bf16_kernel<<<grid_of(T * I / 8, ctx->num_sms), 256, 0, st>>>(gu, T, I, a);
      ZL_LAUNCH_CHECK(ctx);
    } else if (f != ZL_OK) {
      return f;
    }
    if ((s = linear(hb, st, a, L.w_down, x, T, hid, I, true))) return s;
  }
  if (b->num_last > 0) {
    rmsnorm_bf16_kernel<<<(unsigned)b->num_last, 256, 0, st>>>(x, b->last_rows, (const __nv_bfloat16*)m->final_norm,
                                                                hid, m->rms_eps, last);
    ZL_LAUNCH_CHECK(ctx);
    if ((s = linear(hb, st, last, m->lm_head, logits, b->num_last, m->vocab, hid, false, true))) return s;
  }
  return ZL_OK;
}
