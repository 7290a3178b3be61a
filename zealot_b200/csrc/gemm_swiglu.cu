// gemm_swiglu.cu -- the decoder MLP's gate/up projection with the SwiGLU
// activation fused into its epilogue, on the sm_100a tensor cores:
//   out[t][i] = silu(x[t] . w[i]) * (x[t] . w[I + i])
// for x [M][K] bf16 (the normed rows), w [2I][K] bf16 (gate rows, then up
// rows: torch Linear layout of the stacked projection), out [M][I] bf16, fp32
// accumulation. It replaces the reference runner's gate GEMM, up GEMM and
// silu_gate_mul kernel (src/cuda_runner.rs:529-572, src/attention/kernels/
// activation.cu:4-12): the [M][2I] gate/up product is never written to HBM,
// and silu(g) * u is taken from the fp32 accumulators and rounded once.
//
// Persistent kernel, one CTA per SM, output tiles of 128 rows x 128 columns:
//   warp 0      TMA producer: per 64-deep k-block one box of x (128 rows) and
//               two boxes of w (the tile's 128 gate rows and its 128 up rows,
//               stacked into one 256-row B operand), 4-stage ring of 48 KB
//   warp 1      MMA issuer (one thread): per k-block four tcgen05.mma of
//               M = 128, N = 256, K = 16 (kind::f16) into a 256-column TMEM
//               accumulator; two accumulators alternate between tiles so the
//               epilogue of one tile overlaps the products of the next
//   warps 2-5   epilogue, one thread per tile row (TMEM lane): gate columns
//               [0,128) and up columns [128,256) -> silu(g) * u -> bf16 -> HBM
// Tiles are taken m-fastest within a 128-column strip of the output, so the
// CTAs running at one time share a few strips of w through L2 and x (the
// smaller operand) stays L2-resident. Every wait is bounded (status word).
#include "zl_internal.h"
#include "zl_ptx.cuh"

namespace zl {
zl_status make_tmap_bf16(CUtensorMap* map, const void* ptr, uint64_t cols, uint64_t rows,
                         uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows);
}

namespace {

using namespace zl::ptx;

constexpr int BM = 128;                    // rows of x per tile
constexpr int BN = 128;                    // output columns per tile (gate + up: 256 accumulators)
constexpr int BK = 64;                     // k per stage (one 128-byte swizzled row)
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;       // 16 KB
constexpr int B_BYTES = 2 * BN * BK * 2;   // 32 KB
constexpr int STAGE = A_BYTES + B_BYTES;   // 48 KB
constexpr int THREADS = 192;               // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int ACC_COLS = 2 * BN;           // 256 TMEM columns per accumulator

enum Bar { FULL = 0, EMPTY = FULL + STAGES, ACC_FULL = EMPTY + STAGES, ACC_EMPTY = ACC_FULL + 2,
           NUM_BARS = ACC_EMPTY + 2 };

struct Smem {
  static constexpr int kStages = 0;
  static constexpr int kBars = STAGES * STAGE;
  static constexpr int kTmem = kBars + NUM_BARS * 8;
  static constexpr int kTotal = 1024 + kTmem + 16;
};
static_assert(Smem::kTotal <= 232448, "over the 227 KB dynamic shared memory limit");

struct SwigluArgs {
  __nv_bfloat16* out;  // [M][I]
  int* status;
  int M, I, m_blocks, k_blocks, tiles;
};

constexpr uint32_t IDESC = idesc_bf16(BM, 2 * BN, false, false);

// Four MMAs over one 64-deep k-block from one asm block: A and B K-major,
// 128-byte swizzle, k-step kk 32 bytes further along the row (+2 in the
// descriptor's start-address field). acc_first: the first step accumulates.
__device__ __forceinline__ void mma_k64(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t acc_first) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      ".reg .b64 a1, a2, a3, b1, b2, b3;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.eq.b32 q, %4, %4;\n\t"
      "add.s64 a1, %1, 2;\n\t" "add.s64 b1, %2, 2;\n\t"
      "add.s64 a2, %1, 4;\n\t" "add.s64 b2, %2, 4;\n\t"
      "add.s64 a3, %1, 6;\n\t" "add.s64 b3, %2, 6;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a2, b2, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a3, b3, %3, q;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc_first)
      : "memory");
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + __expf(-g)) * u; }

__global__ void __launch_bounds__(THREADS, 1)
gemm_swiglu_kernel(const SwigluArgs a, const __grid_constant__ CUtensorMap tmX,
                   const __grid_constant__ CUtensorMap tmW) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sbase = smem_raw + (base - raw);
  auto bar = [&](int i) { return base + Smem::kBars + 8 * i; };
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(sbase + Smem::kTmem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (aborted(a.status)) return;  // uniform: an earlier launch timed out

  if (threadIdx.x == 0) {
    for (int i = 0; i < NUM_BARS; i++)
      mbar_init(bar(i), (i >= ACC_EMPTY && i < ACC_EMPTY + 2) ? 128 : 1);
    fence_mbar_init();
    prefetch_tmap(&tmX);
    prefetch_tmap(&tmW);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(base + Smem::kTmem, 2 * ACC_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------- producer
    int c = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < a.tiles; tile += gridDim.x) {
      const int m0 = (tile % a.m_blocks) * BM, n0 = (tile / a.m_blocks) * BN;
      for (int kb = 0; kb < a.k_blocks; kb++, c++) {
        const int s = c % STAGES;
        if (!(ok = mbar_wait(bar(EMPTY + s), ((c / STAGES) & 1) ^ 1, a.status))) break;
        const uint32_t dst = base + Smem::kStages + s * STAGE;
        mbar_arrive_expect_tx(bar(FULL + s), STAGE);
        tma_load_2d(dst, &tmX, kb * BK, m0, bar(FULL + s));
        tma_load_2d(dst + A_BYTES, &tmW, kb * BK, n0, bar(FULL + s));                   // gate rows
        tma_load_2d(dst + A_BYTES + BN * BK * 2, &tmW, kb * BK, a.I + n0, bar(FULL + s));  // up rows
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ----------------------------------------------------------- MMA issuer
    int c = 0, it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < a.tiles; tile += gridDim.x, it++) {
      const int buf = it & 1;
      if (!(ok = mbar_wait(bar(ACC_EMPTY + buf), ((it >> 1) & 1) ^ 1, a.status))) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * ACC_COLS;
      for (int kb = 0; kb < a.k_blocks; kb++, c++) {
        const int s = c % STAGES;
        if (!(ok = mbar_wait(bar(FULL + s), (c / STAGES) & 1, a.status))) break;
        tc_fence_after();
        const uint32_t st = base + Smem::kStages + s * STAGE;
        mma_k64(d, sdesc(st, 16, 1024, 2), sdesc(st + A_BYTES, 16, 1024, 2), IDESC, kb > 0 ? 1u : 0u);
        tc_commit(bar(EMPTY + s));
      }
      if (ok) tc_commit(bar(ACC_FULL + buf));
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------- epilogue
    const int q = warp & 3;                       // TMEM lane quadrant of this warp
    const int r = 32 * q + lane;                  // tile row == TMEM lane
    const uint32_t lane_off = (uint32_t)(32 * q) << 16;
    int it = 0;
    for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x, it++) {
      const int buf = it & 1;
      if (!mbar_wait_warp(bar(ACC_FULL + buf), (it >> 1) & 1, a.status)) break;
      tc_fence_after();
      const int m0 = (tile % a.m_blocks) * BM, n0 = (tile / a.m_blocks) * BN;
      const int row = m0 + r;
      const uint32_t acc = tmem + buf * ACC_COLS + lane_off;
      uint4* dst = reinterpret_cast<uint4*>(a.out + (int64_t)row * a.I + n0);
#pragma unroll 1
      for (int c = 0; c < BN / 32; c++) {
        uint32_t g[32], u[32];
        tmem_ld32(acc + 32 * c, g);
        tmem_ld32(acc + BN + 32 * c, u);
        tc_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; i++)
          pk[i] = pack_bf16x2(silu_mul(__uint_as_float(g[2 * i]), __uint_as_float(u[2 * i])),
                              silu_mul(__uint_as_float(g[2 * i + 1]), __uint_as_float(u[2 * i + 1])));
        if (row < a.M) {
#pragma unroll
          for (int i = 0; i < 4; i++)
            dst[4 * c + i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(bar(ACC_EMPTY + buf));  // the MMA thread may overwrite this accumulator
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 2 * ACC_COLS);
  }
}

}  // namespace

namespace zl {

zl_status launch_gemm_swiglu(zl_ctx* ctx, const void* x, const void* w, void* out, int64_t M, int K, int I,
                             cudaStream_t st) {
  if (M <= 0) return ZL_OK;
  if (K <= 0 || K % BK != 0 || I <= 0 || I % BN != 0 || M >= (1ll << 31) || (int64_t)2 * I >= (1ll << 31))
    return ZL_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) & 15)
    return ZL_ERR_UNSUPPORTED;
  const int64_t m_blocks = (M + BM - 1) / BM, n_blocks = I / BN;
  if (m_blocks * n_blocks >= (1ll << 31)) return ZL_ERR_UNSUPPORTED;
  CUtensorMap tx, tw;
  zl_status s = make_tmap_bf16(&tx, x, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK, BM);
  if (s != ZL_OK) return s;
  if ((s = make_tmap_bf16(&tw, w, (uint64_t)K, (uint64_t)2 * I, (uint64_t)K * 2, BK, BN)) != ZL_OK) return s;
  SwigluArgs args;
  args.out = static_cast<__nv_bfloat16*>(out);
  args.status = ctx->d_status;
  args.M = (int)M;
  args.I = I;
  args.m_blocks = (int)m_blocks;
  args.k_blocks = K / BK;
  args.tiles = (int)(m_blocks * n_blocks);
  static std::atomic<uint64_t> attr_set{0};
  if (ctx->device < 64 && !(attr_set.load() & (1ull << ctx->device))) {
    ZL_CUDA_TRY(cudaFuncSetAttribute(gemm_swiglu_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Smem::kTotal));
    attr_set.fetch_or(1ull << ctx->device);
  }
  const int grid = args.tiles < ctx->num_sms ? args.tiles : ctx->num_sms;
  gemm_swiglu_kernel<<<grid, THREADS, Smem::kTotal, st>>>(args, tx, tw);
  ZL_LAUNCH_CHECK(ctx);
  return ZL_OK;
}

}  // namespace zl

extern "C" zl_status zl_linear_swiglu(zl_ctx* ctx, const void* x, const void* w_gate_up, void* out, int64_t M,
                                      int K, int I, zl_stream stream) {
  zl_status s = zl::bind_device(ctx);
  if (s != ZL_OK) return s;
  if (!x || !w_gate_up || !out || M < 0 || K <= 0 || I <= 0)
    return zl::set_error(ZL_ERR_INVALID_ARG, "linear_swiglu: null pointer or bad size");
  s = zl::launch_gemm_swiglu(ctx, x, w_gate_up, out, M, K, I, zl::S(stream));
  if (s == ZL_ERR_UNSUPPORTED)
    return zl::set_error(s, "linear_swiglu: needs K %% 64 == 0, I %% 128 == 0 and 16-byte aligned buffers "
                            "(K=%d, I=%d)", K, I);
  return s;
}
