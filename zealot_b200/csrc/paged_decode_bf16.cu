// paged_decode_bf16.cu -- HBM-bound paged decode attention for bf16 pools,
// head_dim 128, block_size 16, GQA groups of up to 8 query heads.
//
// Replaces paged_attention_kernel / paged_attention_gqa_kernel
// (src/attention/kernels/paged_attention.cu:13-291 of the reference), where
// thread 0 of a CTA did all the math over scalar loads.
//
// Design (B200):
//  * Work is the flat list of (sequence, kv head, 16-token block) triples in
//    (b, kvh, j) order. A persistent grid (one CTA per SM, WARPS warps each)
//    splits that list into equal contiguous ranges, one per warp ("stream-K"
//    at block granularity), so ragged contexts cost no load imbalance.
//  * Each warp runs its own STAGES-deep ring in shared memory: lane 0 issues
//    TMA tile loads (two 64-column boxes per K and per V tile, 128-byte
//    swizzle) that complete on an mbarrier, all lanes consume.
//  * Math on the warp-level tensor-core path: S^T = K * q^T (m16n8k16, the 16
//    tokens of a block are M, the <=8 heads of the group are N), online
//    softmax in registers with warp shuffles, P^T re-laid out by movmatrix,
//    O^T += V^T * P^T with ldmatrix.trans. Every loaded K/V tile serves the
//    whole GQA group. fp32 accumulation.
//  * A (sequence, kv head) that spans several warps is merged by the last
//    warp to finish it (atomic counter in a self-resetting workspace), so
//    there is no second kernel.
#include "zl_internal.h"
#include "zl_ptx.cuh"

#include <cudaTypedefs.h>

#include <mutex>

namespace {

using namespace zl::ptx;

constexpr int D = 128;           // head dim
constexpr int BS = 16;           // tokens per block
constexpr int TILE = BS * D * 2; // bytes of one K (or V) block tile = 4 KB
constexpr int STAGE = 2 * TILE;  // K + V
constexpr int MAX_G = 8;         // query heads per kv head handled per pass
constexpr int MAX_B = 4096;      // sequences per launch (prefix table in smem)
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

// Per-warp partial triple in the workspace.
struct Partial {
  float m[MAX_G];
  float l[MAX_G];
  float o[MAX_G][D];
};

struct DecodeArgs {
  const __nv_bfloat16* q;      // [B][H][D]
  const int32_t* block_tables; // [B][max_blocks]
  const int32_t* seq_lens;     // [B]; in the partial form the end of each token range
  const int32_t* tok_begin;    // partial form: first token of each range (null = 0)
  __nv_bfloat16* out;          // [B][H][D] (normalised form)
  float* m_out;                // partial form: [B][H] max score (natural-log units)
  float* l_out;                // partial form: [B][H] sum of e^(s - m)
  float* o_out;                // partial form: [B][H][D] sum of e^(s - m) v
  Partial* partials;           // [2*W]
  int* counters;               // [0..1] grid barrier words, [2 + b*Hkv + kvh] merge counters;
                               // all zero on entry and exit except the barrier generation
  int* status;
  int B, H, Hkv, G, max_blocks;
  // 1: block_tables / seq_lens / tok_begin are complete before the previous
  // kernel on the stream starts, so they are read before the dependency wait;
  // 0: nothing is read before it.
  int inputs_ahead;
  int64_t num_blocks;
  float scale_log2;            // scale * log2(e)
};

template <int WARPS, int STAGES, bool PARTIAL>
struct Smem {
  static constexpr int kRing = WARPS * STAGES * STAGE;
  static constexpr int kBars = WARPS * STAGES * 8;
  static constexpr int kInfo = WARPS * STAGES * 4;
  static constexpr int kPrefix = (MAX_B + 1) * 4;
  static constexpr int kJbase = PARTIAL ? MAX_B * 4 : 0;  // table index of each range's first block
  static constexpr int kParts = (kRing + kBars + kInfo + kPrefix + kJbase + 15) & ~15;
  static constexpr int kPartBytes = WARPS * (2 * MAX_G + MAX_G * D) * 4;  // the warps' staged shares
  static constexpr int kTotal = 1024 /*alignment slack*/ + kParts + kPartBytes;
};

// Blocks of sequence b's token range and the block-table index of its first
// block. The normalised form attends to [0, seq_lens[b]); the partial form to
// [tok_begin[b], seq_lens[b]). `over` is set when the range runs past the
// table (the blocks past it are dropped).
template <bool PARTIAL>
__device__ __forceinline__ int range_blocks(const DecodeArgs& a, int b, int& jt0, bool& over) {
  const int e = max(a.seq_lens[b], 0);
  int s = 0;
  if (PARTIAL && a.tok_begin) s = max(a.tok_begin[b], 0);
  jt0 = s / BS;
  int j1 = (e + BS - 1) / BS;
  over = j1 > a.max_blocks;
  if (over) j1 = a.max_blocks;
  return s < e ? max(j1 - jt0, 0) : 0;
}

// Swizzled byte offset of (row r, 16-byte chunk c in 0..15) inside a K or V
// tile: two 2 KB boxes of [16 rows][64 cols], 128-byte swizzle (chunk ^= row%8).
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
  return (uint32_t)((c >> 3) * 2048 + r * 128 + ((((c & 7) ^ (r & 7))) << 4));
}

// Whether any of the n int32 entries at p is negative; all `nthreads` threads
// of the CTA call it and share the loads (16-byte loads between a scalar head
// and tail).
__device__ __forceinline__ bool any_negative(const int32_t* p, int n, int tid, int nthreads) {
  const int head = min(n, (int)(((16 - (reinterpret_cast<uintptr_t>(p) & 15)) & 15) >> 2));
  bool neg = tid < head && __ldg(p + tid) < 0;
  const int4* p4 = reinterpret_cast<const int4*>(p + head);
  const int n4 = (n - head) >> 2;
#pragma unroll 4
  for (int i = tid; i < n4; i += nthreads) {
    const int4 v = __ldg(p4 + i);
    neg |= (v.x | v.y | v.z | v.w) < 0;
  }
  const int tail = head + 4 * n4 + tid;
  if (tail < n) neg |= __ldg(p + tail) < 0;
  return neg;
}

// Output of a merged (sequence, head) row: lane L holds elements [4L, 4L+4)
// of the weighted sum `num` and the row's weight total `den` (relative to the
// maximum M over the contributors). The normalised form stores num / den in
// bf16; the partial form stores the triple (M, den, num).
template <bool PARTIAL>
__device__ __forceinline__ void emit_merged(const DecodeArgs& a, int64_t row, int lane, float M,
                                            float den, float4 num) {
  if constexpr (PARTIAL) {
    if (lane == 0) { a.m_out[row] = M; a.l_out[row] = den; }
    reinterpret_cast<float4*>(a.o_out + row * D)[lane] = num;
  } else {
    const float inv = den > 0.f ? 1.f / den : 0.f;
    __nv_bfloat162 lo = __floats2bfloat162_rn(num.x * inv, num.y * inv);
    __nv_bfloat162 hi = __floats2bfloat162_rn(num.z * inv, num.w * inv);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&lo);
    pk.y = *reinterpret_cast<uint32_t*>(&hi);
    reinterpret_cast<uint2*>(a.out + row * D)[lane] = pk;
  }
}

// Warp partial of one (sequence, kv head) segment, staged in shared memory for
// the CTA's combine: m in natural-log units, l and o relative to it.
struct WarpPart {
  float m[MAX_G];
  float l[MAX_G];
  float o[MAX_G][D];
};

// Unit (warp or CTA) owning flat block x when the flat list is split into
// contiguous ranges of `per` or `per + 1` blocks (the first `rem` units take
// one more).
__device__ __forceinline__ int owner_unit(int x, int per, int rem) {
  const int big = rem * (per + 1);
  return x < big ? x / (per + 1) : rem + (x - big) / per;
}
__device__ __forceinline__ int unit_start(int u, int per, int rem) { return u * per + min(u, rem); }

// Named barrier over the CTA's WARPS warps (id 1; __syncthreads is id 0).
template <int WARPS>
__device__ __forceinline__ void cta_bar() {
  asm volatile("bar.sync 1, %0;" ::"r"(WARPS * 32) : "memory");
}

// Per-warp ranges are used while a segment spreads over fewer than
// kGroupAvgContrib warps on average and over at most kMaxWarpContrib warps;
// beyond that the CTA's warps share one range (fewer, larger merges). Measured
// on B200 (C2 shapes): per-warp ranges win at about 2-3 contributors per
// segment, CTA ranges from about 5.
constexpr int kGroupAvgContrib = 4;
constexpr int kMaxWarpContrib = 16;

// Merges the partial triples of `nc` consecutive units for head n of a split
// segment (m natural-log, l, o relative to m) and emits the row; one warp.
template <bool PARTIAL, typename SlotOf>
__device__ __forceinline__ void merge_units(const DecodeArgs& a, int64_t row, int n, int nc, int lane,
                                            SlotOf slot_of) {
  float M = -INFINITY;
  for (int k0 = 0; k0 < nc; k0 += 32)
    if (k0 + lane < nc) M = fmaxf(M, __ldcg(&slot_of(k0 + lane)->m[n]));
#pragma unroll
  for (int off = 16; off; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float den = 0.f;
  float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k0 = 0; k0 < nc; k0 += 32) {
    float wl = 0.f;
    if (k0 + lane < nc) {
      const Partial* pc = slot_of(k0 + lane);
      const float mc = __ldcg(&pc->m[n]);
      wl = (mc == -INFINITY) ? 0.f : __expf(mc - M);
      den += wl * __ldcg(&pc->l[n]);
    }
    const int cnt = min(32, nc - k0);
    for (int u0 = 0; u0 < cnt; u0 += 8) {
      float4 x[8];
#pragma unroll
      for (int u = 0; u < 8; u++)  // eight rows in flight
        x[u] = (u0 + u < cnt) ? __ldcg(reinterpret_cast<const float4*>(slot_of(k0 + u0 + u)->o[n]) + lane)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const float w = __shfl_sync(0xffffffffu, wl, (u0 + u) & 31);
        if (u0 + u < cnt) {
          num.x += w * x[u].x; num.y += w * x[u].y; num.z += w * x[u].z; num.w += w * x[u].w;
        }
      }
    }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
  emit_merged<PARTIAL>(a, row, lane, M, den, num);
}

// The same merge for all G heads of the segment at once (one warp): lane c
// holds contributor c's (m, l) for every head, and the rows of contributors 0
// and 1 are loaded in the same round, so a split over two contributors (the
// common case of per-warp ranges) costs one L2 round trip before the math.
template <bool PARTIAL, typename SlotOf>
__device__ __forceinline__ void merge_units_all(const DecodeArgs& a, int64_t row0, int G, int nc, int lane,
                                                SlotOf slot_of) {
  float M[MAX_G], den[MAX_G], mc[MAX_G], lc[MAX_G];
  float4 x1[MAX_G], x2[MAX_G];
  {
    const bool mine = lane < nc;
    const Partial* pc = slot_of(mine ? lane : 0);
    const float4* o1 = reinterpret_cast<const float4*>(&slot_of(0)->o[0][0]) + lane;
    const float4* o2 = reinterpret_cast<const float4*>(&slot_of(nc > 1 ? 1 : 0)->o[0][0]) + lane;
#pragma unroll
    for (int n = 0; n < MAX_G; n++) {
      mc[n] = -INFINITY;
      lc[n] = 0.f;
      if (n < G) {
        if (mine) { mc[n] = __ldcg(&pc->m[n]); lc[n] = __ldcg(&pc->l[n]); }
        x1[n] = __ldcg(o1 + n * (D / 4));
        x2[n] = __ldcg(o2 + n * (D / 4));
      }
    }
  }
#pragma unroll
  for (int n = 0; n < MAX_G; n++) { M[n] = mc[n]; den[n] = 0.f; }
  // contributors past 32 (very long sequences): their maxima too
  for (int c0 = 32; c0 < nc; c0 += 32)
    if (c0 + lane < nc) {
      const Partial* pc = slot_of(c0 + lane);
#pragma unroll
      for (int n = 0; n < MAX_G; n++)
        if (n < G) M[n] = fmaxf(M[n], __ldcg(&pc->m[n]));
    }
#pragma unroll
  for (int n = 0; n < MAX_G; n++)
#pragma unroll
    for (int off = 16; off; off >>= 1) M[n] = fmaxf(M[n], __shfl_xor_sync(0xffffffffu, M[n], off));
  float4 num[MAX_G];
#pragma unroll
  for (int n = 0; n < MAX_G; n++) num[n] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int c0 = 0; c0 < nc; c0 += 32) {
    float wl[MAX_G];
    if (c0 + lane < nc) {
      const Partial* pc = slot_of(c0 + lane);
#pragma unroll
      for (int n = 0; n < MAX_G; n++) {
        wl[n] = 0.f;
        if (n < G) {
          const float m_ = c0 == 0 ? mc[n] : __ldcg(&pc->m[n]);
          const float l_ = c0 == 0 ? lc[n] : __ldcg(&pc->l[n]);
          wl[n] = (m_ == -INFINITY) ? 0.f : __expf(m_ - M[n]);
          den[n] += wl[n] * l_;
        }
      }
    } else {
#pragma unroll
      for (int n = 0; n < MAX_G; n++) wl[n] = 0.f;
    }
    const int cnt = min(32, nc - c0);
    for (int k = 0; k < cnt; k += 2) {
      const bool second = k + 1 < cnt;
      if (c0 + k > 0) {  // rows of contributors 0 and 1 are already loaded
        const float4* o1 = reinterpret_cast<const float4*>(&slot_of(c0 + k)->o[0][0]) + lane;
        const float4* o2 = reinterpret_cast<const float4*>(&slot_of(c0 + k + (second ? 1 : 0))->o[0][0]) + lane;
#pragma unroll
        for (int n = 0; n < MAX_G; n++) {
          if (n < G) {
            x1[n] = __ldcg(o1 + n * (D / 4));
            x2[n] = __ldcg(o2 + n * (D / 4));
          }
        }
      }
#pragma unroll
      for (int n = 0; n < MAX_G; n++) {
        const float w1 = __shfl_sync(0xffffffffu, wl[n], k);
        const float w2 = second ? __shfl_sync(0xffffffffu, wl[n], k + 1) : 0.f;
        if (n < G) {
          num[n].x += w1 * x1[n].x + w2 * x2[n].x;
          num[n].y += w1 * x1[n].y + w2 * x2[n].y;
          num[n].z += w1 * x1[n].z + w2 * x2[n].z;
          num[n].w += w1 * x1[n].w + w2 * x2[n].w;
        }
      }
    }
  }
#pragma unroll
  for (int n = 0; n < MAX_G; n++) {
#pragma unroll
    for (int off = 16; off; off >>= 1) den[n] += __shfl_xor_sync(0xffffffffu, den[n], off);
    if (n < G) emit_merged<PARTIAL>(a, row0 + n, lane, M[n], den[n], num[n]);
  }
}

// PARTIAL = false: normalised bf16 output over [0, seq_lens[b]).
// PARTIAL = true: the unnormalised triple (m, l, o) of each (sequence, head)
// over the token range [tok_begin[b], seq_lens[b]), m being the true maximum
// score (the sequence-split form, merged across GPUs afterwards).
//
// Work split. The flat list of (sequence, kv head, 16-token block) in
// (b, kvh, j) order is cut into equal contiguous ranges, one per unit
// ("stream-K" at block granularity, so ragged contexts cost no imbalance). The
// kernel picks the unit from the job it finds (the same choice in every CTA):
//  * per-warp ranges for long jobs: warps stream independently; a segment
//    (sequence, kv head) inside one warp's range is written out directly, a
//    segment spanning warps leaves one partial per warp and the last warp to
//    finish merges them;
//  * per-CTA ranges for short jobs: warp w of a CTA takes blocks w, w + WARPS,
//    ... of the CTA's range, at each segment end the warps' partials are
//    combined through shared memory (CTA barrier), and a segment spanning CTAs
//    is merged by the last CTA to finish it -- a few large merges instead of
//    many small ones.
template <int WARPS, int STAGES, bool PARTIAL>
__global__ void __launch_bounds__(WARPS * 32, 1)
paged_decode_bf16_kernel(const DecodeArgs a, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV) {
  using SM = Smem<WARPS, STAGES, PARTIAL>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_u32 - raw_u32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + SM::kRing);
  int* info = reinterpret_cast<int*>(base + SM::kRing + SM::kBars);
  int* prefix = reinterpret_cast<int*>(base + SM::kRing + SM::kBars + SM::kInfo);
  int* jbase = reinterpret_cast<int*>(base + SM::kRing + SM::kBars + SM::kInfo + SM::kPrefix);
  WarpPart* wpart = reinterpret_cast<WarpPart*>(base + SM::kParts);
  __shared__ int s_last;
  __shared__ int s_max_nb;    // longest sequence in blocks
  __shared__ int s_nonempty;  // sequences with at least one block

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int B = a.B, Hkv = a.Hkv;

  // Programmatic dependent launch: the next kernel may be scheduled now; this
  // one waits for its predecessor before the first read of anything that
  // kernel could write (at once, unless the caller declared the tables and
  // lengths ready ahead: then after the prologue and the first table reads).
  griddep_launch_dependents();
  if (!a.inputs_ahead) griddep_wait();
  // An earlier launch timed out and was not cleared: return, the whole CTA
  // alike (its warps may meet at CTA barriers further on).
  if (__syncthreads_or(aborted(a.status))) return;
  if (tid == 0) {
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    s_max_nb = 0;
    s_nonempty = 0;
  }
  for (int i = tid; i < WARPS * STAGES; i += blockDim.x) mbar_init(smem_u32(&bars[i]), 1);

  // ---- per-CTA prologue: prefix[b] = sum_{b'<b} nblk(b') (flat start of b is Hkv * prefix[b])
  {
    constexpr int T = WARPS * 32;
    const int per = (B + T - 1) / T;
    const int b0 = tid * per;
    int local = 0, lmax = 0, lcount = 0;
    for (int k = 0; k < per; k++) {
      const int b = b0 + k;
      if (b < B) {
        int jt0;
        bool over;
        const int nb = range_blocks<PARTIAL>(a, b, jt0, over);
        if (over && blockIdx.x == 0) atomicOr(a.status, ZL_DEV_OOB);
        if (PARTIAL) jbase[b] = jt0;
        local += nb;
        lmax = max(lmax, nb);
        lcount += nb > 0;
      }
    }
    // block-wide exclusive scan of `local`
    int incl = local;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    __shared__ int warp_tot[WARPS];
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();  // (also orders s_max_nb = 0 before the atomicMax below)
    if (lmax > 0) {
      atomicMax(&s_max_nb, lmax);
      atomicAdd(&s_nonempty, lcount);
    }
    int run = incl - local;
    for (int w = 0; w < warp; w++) run += warp_tot[w];
    if (tid == 0) prefix[0] = 0;
    for (int k = 0; k < per; k++) {
      const int b = b0 + k;
      if (b < B) {
        int jt0;
        bool over;
        run += range_blocks<PARTIAL>(a, b, jt0, over);
        prefix[b + 1] = run;
      }
    }
  }
  fence_mbar_init();
  __syncthreads();

  const int TB = prefix[B] * Hkv;  // flat work items (< 2^31, checked on the host)

  // Sequences with no context produce zeros, (-inf, 0, 0) in the partial
  // form (CTA 0 writes them).
  if (blockIdx.x == 0) {
    griddep_wait();
    for (int b = warp; b < B; b += WARPS) {
      if (prefix[b + 1] == prefix[b]) {
        if constexpr (PARTIAL) {
          for (int i = lane; i < a.H; i += 32) {
            a.m_out[(int64_t)b * a.H + i] = -INFINITY;
            a.l_out[(int64_t)b * a.H + i] = 0.f;
          }
          const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int i = lane; i < a.H * D / 4; i += 32)
            reinterpret_cast<float4*>(a.o_out + (int64_t)b * a.H * D)[i] = z;
        } else {
          uint2 z = make_uint2(0, 0);
          for (int i = lane; i < a.H * D / 4; i += 32)
            reinterpret_cast<uint2*>(a.out + (int64_t)b * a.H * D)[i] = z;
        }
      }
    }
  }
  if (TB == 0) return;

  // ---- the unit of the split, the same in every CTA
  const int nwarps = (int)gridDim.x * WARPS;
  bool grouped;
  {
    const int per_warp = TB / min(nwarps, TB);
    const int avg_nb = prefix[B] / max(s_nonempty, 1);
    grouped = avg_nb >= (kGroupAvgContrib - 1) * per_warp ||
              (s_max_nb + per_warp - 1) / per_warp + 1 > kMaxWarpContrib;
  }
  // Active units: never more than work items, so every active unit owns at
  // least one block and the contributors of a split segment are the
  // consecutive units owner_unit(first block) .. owner_unit(last block).
  const int U = min(grouped ? (int)gridDim.x : nwarps, TB);
  const int unit = grouped ? (int)blockIdx.x : (int)blockIdx.x * WARPS + warp;
  if (grouped && unit >= U) return;  // uniform over the CTA
  const int uper = TB / U, urem = TB - uper * U;
  const bool active = unit < U;      // per-warp: warps past U own nothing
  const int u0 = active ? unit_start(unit, uper, urem) : TB;
  const int u1 = active ? u0 + uper + (unit < urem ? 1 : 0) : TB;
  // this warp's items: flat blocks u0 + ioff + istride * k, k in [0, nwork)
  const int istride = grouped ? WARPS : 1, ioff = grouped ? warp : 0;
  const int nwork = u1 - u0 > ioff ? (u1 - u0 - ioff + istride - 1) / istride : 0;
  auto item_flat = [&](int k) { return u0 + ioff + istride * k; };

  // Segment of flat block f: sequence b (largest with Hkv*prefix[b] <= f), kv
  // head and block index j inside the segment.
  auto locate = [&](int f, int& b, int& kvh, int& j) {
    int lo = 0, hi = B;  // Hkv*prefix[lo] <= f < Hkv*prefix[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (prefix[mid] * Hkv <= f) lo = mid; else hi = mid;
    }
    while (prefix[lo + 1] * Hkv <= f) lo++;  // skip empty sequences (prefix equal)
    b = lo;
    const int nb = prefix[b + 1] - prefix[b];
    const int off = f - prefix[b] * Hkv;
    kvh = off / nb;
    j = off - kvh * nb;
  };

  // Partial form: a negative table entry before a range's start ends the
  // sequence before the range, which then holds no tokens. The CTA scans the
  // entries [0, jbase[b]) of every sequence its warps touch, once, and marks a
  // sequence so found in the sign bit of jbase[b].
  if constexpr (PARTIAL) {
    const int f_lo = grouped ? u0 : unit_start(blockIdx.x * WARPS, uper, urem);
    const int w_hi = min((int)(blockIdx.x + 1) * WARPS, U);
    const int f_hi = grouped ? u1 : (w_hi > (int)blockIdx.x * WARPS ? unit_start(w_hi, uper, urem) : f_lo);
    if (f_hi > f_lo) {  // uniform over the CTA
      int bl, bh, k_, j_;
      locate(f_lo, bl, k_, j_);
      locate(f_hi - 1, bh, k_, j_);
      for (int b = bl; b <= bh; b++) {
        const int n = jbase[b];
        bool neg = false;
        if (n > 0) neg = any_negative(a.block_tables + (int64_t)b * a.max_blocks, n, tid, WARPS * 32);
        if (__syncthreads_or(neg) && tid == 0) jbase[b] = n | (int)0x80000000;
      }
    }
    __syncthreads();
  }
  auto table_base = [&](int b) -> int { return PARTIAL ? (jbase[b] & 0x7fffffff) : 0; };
  auto cut_before = [&](int b) -> bool { return PARTIAL && jbase[b] < 0; };

  const uint32_t ring = base_u32 + warp * STAGES * STAGE;
  uint64_t* wbars = bars + warp * STAGES;
  int* winfo = info + warp * STAGES;
  const uint64_t policy = policy_evict_first();

  // ---------------- producer: item list in chunks of 32 (warp-wide) ----------------
  // Every 32 items the whole warp resolves the next 32 at once: lane L holds
  // the TMA row and the valid tokens of item ch_base + L. A negative table
  // entry ends its sequence (paged_attention.cu:66-67): a block is dropped when
  // any entry at or before it in the same sequence is negative. Each lane
  // checks its own entry and, in the CTA split, the WARPS - 1 entries before
  // it (the blocks the CTA's other warps take), so the lanes' windows tile the
  // table; the ballot carries the result along the chunk and carry_seg /
  // carry_trunc across chunks, and the first item's earlier entries are
  // scanned once.
  const int32_t* const tables = a.block_tables;
  // ch_end: one past the current chunk's last item; p_hi: one past the last
  // item produced (a timed-out warp drains up to it)
  int ch_base = -32, ch_end = 0, ch_y = 0, ch_nv = 0, p_hi = 0;
  int carry_seg = -1, carry_trunc = 0;
  if (nwork > 0) {
    int b, kvh, j;
    locate(item_flat(0), b, kvh, j);
    const int t_lo = table_base(b);
    j += t_lo;
    bool neg = cut_before(b);
    const int32_t* tb = tables + (int64_t)b * a.max_blocks;
    // eight independent loads per lane in flight: one memory latency for the
    // first 256 entries instead of one per 32
    for (int t0 = t_lo; t0 < j; t0 += 256) {
      int v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int t = t0 + 32 * u + lane;
        v[u] = t < j ? __ldg(tb + t) : 0;
      }
#pragma unroll
      for (int u = 0; u < 8; u++) neg |= v[u] < 0;
    }
    carry_trunc = __any_sync(0xffffffffu, neg) ? 1 : 0;
    carry_seg = b * Hkv + kvh;
  }
  // A chunk's table entries and lengths are fetched one chunk ahead (the f_
  // registers) and resolved when the producer reaches the chunk, so the
  // loads' latency hides behind the current chunk's 32 items.
  int f_seg = -1, f_e = 0, f_b = 0, f_kvh = 0, f_j = 0, f_len = 0, f_beg = 0;
  bool f_wneg = false;
  auto fetch_chunk = [&](int cbase) {
    const int idx = cbase + lane;
    f_seg = -1; f_e = 0; f_b = 0; f_kvh = 0; f_j = 0; f_len = 0; f_beg = 0;
    f_wneg = false;
    if (idx < nwork) {
      int b, kvh, j;
      locate(item_flat(idx), b, kvh, j);
      f_seg = b * Hkv + kvh;
      const int32_t* tb = tables + (int64_t)b * a.max_blocks;
      const int t = table_base(b) + j;  // table index from here on
      f_e = tb[t];
      // the other warps' blocks between this warp's previous item and this one
      for (int u = 1; u < istride; u++)
        if (j >= u) f_wneg |= tb[t - u] < 0;
      f_len = a.seq_lens[b];  // issued with the table reads: one latency, not two
      if constexpr (PARTIAL) f_beg = a.tok_begin ? a.tok_begin[b] : 0;
      f_b = b;
      f_kvh = kvh;
      f_j = t;
    }
  };
  auto build_chunk = [&](int cbase) {
    const int idx = cbase + lane;
    const bool ok = idx < nwork;
    const int seg = f_seg, e = f_e, b = f_b, kvh = f_kvh, j = f_j, len = f_len, beg = f_beg;
    const bool wneg = f_wneg;
    (void)b; (void)beg;
    const unsigned negm = __ballot_sync(0xffffffffu, ok && (e < 0 || wneg));
    const int prev = __shfl_up_sync(0xffffffffu, seg, 1);
    const unsigned startm = __ballot_sync(0xffffffffu, lane == 0 || seg != prev);
    const unsigned upto = lane == 31 ? 0xffffffffu : ((2u << lane) - 1u);
    const int my_start = 31 - __clz(startm & upto);
    bool trunc = (negm & upto & ~((1u << my_start) - 1u)) != 0;
    if (my_start == 0 && seg == carry_seg && carry_trunc) trunc = true;
    if (ok && cut_before(b)) trunc = true;
    int nv = 0, y = 0;
    if (ok && !trunc) {
      if ((int64_t)e >= a.num_blocks) {
        atomicOr(a.status, ZL_DEV_OOB);
      } else {
        // valid tokens [lo, hi) of the block; nv packs hi | lo << 8
        const int hi = min(len - j * BS, BS);
        const int lo = PARTIAL ? max(beg - j * BS, 0) : 0;
        nv = hi | (lo << 8);
        y = (int)(((int64_t)e * Hkv + kvh) * BS);
      }
    }
    const int last = min(31, nwork - 1 - cbase);
    carry_seg = __shfl_sync(0xffffffffu, seg, last);
    carry_trunc = __shfl_sync(0xffffffffu, trunc ? 1 : 0, last);
    ch_base = cbase;
    ch_end = min(cbase + 32, nwork);
    ch_y = y;
    ch_nv = nv;
    if (cbase + 32 < nwork) fetch_chunk(cbase + 32);
  };
  // Issue the loads of item i of this warp into its ring slot (all lanes
  // call; lane 0 issues).
  auto produce = [&](int i) {
    if (i >= nwork) return;
    if (i >= ch_end) build_chunk(i & ~31);
    p_hi = i + 1;
    const int src = i - ch_base;
    const int y = __shfl_sync(0xffffffffu, ch_y, src);
    const int nvalid = __shfl_sync(0xffffffffu, ch_nv, src);
    if (lane == 0) {
      const int slot = i % STAGES;
      winfo[slot] = nvalid;
      const uint32_t bar = smem_u32(&wbars[slot]);
      if (nvalid > 0) {
        const uint32_t dst = ring + slot * STAGE;
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(bar, STAGE);
        tma_load_2d_hint(dst, &tmK, 0, y, bar, policy);
        tma_load_2d_hint(dst + 2048, &tmK, 64, y, bar, policy);
        tma_load_2d_hint(dst + TILE, &tmV, 0, y, bar, policy);
        tma_load_2d_hint(dst + TILE + 2048, &tmV, 64, y, bar, policy);
      } else {
        mbar_arrive(bar);
      }
    }
  };

  if (nwork > 0) {  // the first 32 items' table entries (and the next 32 fetched)
    fetch_chunk(0);
    build_chunk(0);
  }
  griddep_wait();  // K/V, q and the outputs belong to the stream order from here on
  {
    const int pre = min(nwork, STAGES);
    for (int k = 0; k < pre; k++) produce(k);
  }
  __syncwarp();
  if (!active) return;  // a per-warp split's idle warp (no CTA barriers in that split)

  // ---------------- consumer state (all lanes) ----------------
  int cb, ckvh, cj_;
  locate(u0, cb, ckvh, cj_);
  const int quad = lane >> 2;   // 0..7 : token row (S), head column (B operand)
  const int qid = lane & 3;     // 0..3
  const int mat = lane >> 3, mrow = lane & 7;
  // this lane's ldmatrix row addresses inside a K / V tile (swizzled)
  uint32_t kofs[8], vofs[8];
#pragma unroll
  for (int t = 0; t < 8; t++) {
    kofs[t] = tile_off(mrow + ((mat & 1) << 3), 2 * t + (mat >> 1));
    vofs[t] = tile_off(mrow + ((mat >> 1) << 3), 2 * t + (mat & 1));
  }
  // The running max only moves when a score exceeds it by more than 2^8: until
  // then p = 2^(s - m) <= 256 stays exact enough in bf16 and fp32, and the
  // block needs neither the max reduction nor the O rescale.
  constexpr float kLazy = 8.f;
  bool timed_out = false;
  int i_fail = 0;  // first item not consumed after a timed-out wait
  const int G = a.G;

  // q of the next segment, loaded while the current one streams
  uint32_t qn[8][2];
  int qn_seg = -1;
  const bool hv = quad < G;
  auto load_q = [&](int qb, int qh0, uint32_t (&dst)[8][2]) {
    const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
        a.q + ((int64_t)qb * a.H + qh0 + (hv ? quad : 0)) * D);
#pragma unroll
    for (int ks = 0; ks < 8; ks++) {
      dst[ks][0] = hv ? __ldg(qrow + ks * 8 + qid) : 0u;
      dst[ks][1] = hv ? __ldg(qrow + ks * 8 + 4 + qid) : 0u;
    }
  };

  // Segments of the unit's range, in order. In the CTA split every warp of
  // the CTA visits each of them (the combine's CTA barriers need it), whether
  // or not the warp has items there.
  int i = 0;  // next item of this warp
  for (;;) {
    const int nb = prefix[cb + 1] - prefix[cb];
    const int seg_S = prefix[cb] * Hkv + ckvh * nb;
    const int seg_E = seg_S + nb;
    const int hi = min(seg_E, u1);
    const int k_end = min(nwork, (hi - u0 - ioff + istride - 1) / istride);
    const int head0 = ckvh * G;
    const bool whole = seg_S >= u0 && seg_E <= u1;
    const int e_slot = (seg_S <= u0 && u0 < seg_E) ? 0 : 1;  // the range's first or last segment

    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float tm0 = -INFINITY, tm1 = -INFINITY;  // true maxima (partial form)
    float o[8][4];
#pragma unroll
    for (int t = 0; t < 8; t++) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;

    if (i < k_end) {
      uint32_t qf[8][2];
      if (qn_seg == cb * Hkv + ckvh) {
#pragma unroll
        for (int ks = 0; ks < 8; ks++) { qf[ks][0] = qn[ks][0]; qf[ks][1] = qn[ks][1]; }
      } else {
        load_q(cb, head0, qf);
      }
      qn_seg = -1;
      if (k_end < nwork) {  // this warp's items continue into the next non-empty segment
        int nbq = cb, nkq = ckvh + 1;
        if (nkq == Hkv) {
          nkq = 0;
          do { nbq++; } while (nbq < B && prefix[nbq + 1] == prefix[nbq]);
        }
        if (nbq < B) {
          load_q(nbq, nkq * G, qn);
          qn_seg = nbq * Hkv + nkq;
        }
      }

      // Two items per step: their K/V tiles feed interleaved MMA chains and
      // share one softmax / rescale decision. A step whose second item is
      // missing (odd count) or skipped reads the valid block's tile for both
      // with the missing one fully masked, so no unloaded tile is read.
      while (i < k_end) {
        const bool two = i + 1 < k_end;
        const int step = two ? 2 : 1;
        if (timed_out) {  // keep the visiting order; no more loads or math
          i += step;
          continue;
        }
        const int slotA = i % STAGES;
        if (!mbar_wait_warp(smem_u32(&wbars[slotA]), (uint32_t)((i / STAGES) & 1), a.status)) {
          timed_out = true;
          i_fail = i;
          continue;
        }
        int slotB = slotA, nvB = 0, loB = 0;
        const int infoA = winfo[slotA];
        const int nvA = infoA & 0xff, loA = PARTIAL ? (infoA >> 8) : 0;
        if (two) {
          slotB = (i + 1) % STAGES;
          if (!mbar_wait_warp(smem_u32(&wbars[slotB]), (uint32_t)(((i + 1) / STAGES) & 1), a.status)) {
            timed_out = true;
            i_fail = i;
            continue;
          }
          const int infoB = winfo[slotB];
          nvB = infoB & 0xff;
          if constexpr (PARTIAL) loB = infoB >> 8;
        }
        if (nvA > 0 || nvB > 0) {
          uint32_t kA = ring + slotA * STAGE, kB = ring + slotB * STAGE;
          if (nvA == 0) kA = kB;
          if (nvB == 0) kB = kA;
          // zero V rows outside the valid tokens so 0 * garbage cannot be NaN
          if (nvA > 0 && nvA < BS) {
            uint8_t* vt = base + (kA + TILE - base_u32);
            for (int x = lane; x < (BS - nvA) * 16; x += 32) {
              const int r = nvA + (x >> 4), c = x & 15;
              *reinterpret_cast<uint4*>(vt + tile_off(r, c)) = make_uint4(0, 0, 0, 0);
            }
          }
          if (nvB > 0 && nvB < BS) {
            uint8_t* vt = base + (kB + TILE - base_u32);
            for (int x = lane; x < (BS - nvB) * 16; x += 32) {
              const int r = nvB + (x >> 4), c = x & 15;
              *reinterpret_cast<uint4*>(vt + tile_off(r, c)) = make_uint4(0, 0, 0, 0);
            }
          }
          if constexpr (PARTIAL) {  // rows before the range start
            if (nvA > 0 && loA > 0) {
              uint8_t* vt = base + (kA + TILE - base_u32);
              for (int x = lane; x < loA * 16; x += 32)
                *reinterpret_cast<uint4*>(vt + tile_off(x >> 4, x & 15)) = make_uint4(0, 0, 0, 0);
            }
            if (nvB > 0 && loB > 0) {
              uint8_t* vt = base + (kB + TILE - base_u32);
              for (int x = lane; x < loB * 16; x += 32)
                *reinterpret_cast<uint4*>(vt + tile_off(x >> 4, x & 15)) = make_uint4(0, 0, 0, 0);
            }
          }
          __syncwarp();
          // S^T = K q^T for both blocks, four independent chains
          float sA[4] = {0.f, 0.f, 0.f, 0.f}, sA2[4] = {0.f, 0.f, 0.f, 0.f};
          float sB[4] = {0.f, 0.f, 0.f, 0.f}, sB2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int ks = 0; ks < 8; ks += 2) {
            uint32_t a0, a1, a2, a3, b0, b1, b2, b3, c0_, c1_, c2_, c3_, d0, d1, d2, d3;
            ldsm_x4(kA + kofs[ks], a0, a1, a2, a3);
            ldsm_x4(kB + kofs[ks], b0, b1, b2, b3);
            ldsm_x4(kA + kofs[ks + 1], c0_, c1_, c2_, c3_);
            ldsm_x4(kB + kofs[ks + 1], d0, d1, d2, d3);
            mma_bf16_16816(sA, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
            mma_bf16_16816(sB, b0, b1, b2, b3, qf[ks][0], qf[ks][1]);
            mma_bf16_16816(sA2, c0_, c1_, c2_, c3_, qf[ks + 1][0], qf[ks + 1][1]);
            mma_bf16_16816(sB2, d0, d1, d2, d3, qf[ks + 1][0], qf[ks + 1][1]);
          }
          // mask + scale to log2 units
          const float sc = a.scale_log2;
          const bool va0 = quad < nvA && quad >= loA, va1 = quad + 8 < nvA && quad + 8 >= loA;
          const bool vb0 = quad < nvB && quad >= loB, vb1 = quad + 8 < nvB && quad + 8 >= loB;
          sA[0] = va0 ? (sA[0] + sA2[0]) * sc : -INFINITY;
          sA[1] = va0 ? (sA[1] + sA2[1]) * sc : -INFINITY;
          sA[2] = va1 ? (sA[2] + sA2[2]) * sc : -INFINITY;
          sA[3] = va1 ? (sA[3] + sA2[3]) * sc : -INFINITY;
          sB[0] = vb0 ? (sB[0] + sB2[0]) * sc : -INFINITY;
          sB[1] = vb0 ? (sB[1] + sB2[1]) * sc : -INFINITY;
          sB[2] = vb1 ? (sB[2] + sB2[2]) * sc : -INFINITY;
          sB[3] = vb1 ? (sB[3] + sB2[3]) * sc : -INFINITY;
          const float c0m = fmaxf(fmaxf(sA[0], sA[2]), fmaxf(sB[0], sB[2]));
          const float c1m = fmaxf(fmaxf(sA[1], sA[3]), fmaxf(sB[1], sB[3]));
          if constexpr (PARTIAL) { tm0 = fmaxf(tm0, c0m); tm1 = fmaxf(tm1, c1m); }
          const bool grow = c0m > m0 + kLazy || c1m > m1 + kLazy;
          if (__any_sync(0xffffffffu, grow)) {
            float bm0 = c0m, bm1 = c1m;
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
              bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, off));
              bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, off));
            }
            const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
            const float al0 = (m0 == -INFINITY) ? 0.f : ex2(m0 - mn0);
            const float al1 = (m1 == -INFINITY) ? 0.f : ex2(m1 - mn1);
            m0 = mn0; m1 = mn1;
            l0 *= al0; l1 *= al1;
#pragma unroll
            for (int t = 0; t < 8; t++) {
              o[t][0] *= al0; o[t][1] *= al1; o[t][2] *= al0; o[t][3] *= al1;
            }
          }
          float pA[4], pB[4];
#pragma unroll
          for (int r = 0; r < 4; r++) {
            const float mr = (r & 1) ? m1 : m0;
            pA[r] = sA[r] == -INFINITY ? 0.f : ex2(sA[r] - mr);
            pB[r] = sB[r] == -INFINITY ? 0.f : ex2(sB[r] - mr);
          }
          l0 += (pA[0] + pA[2]) + (pB[0] + pB[2]);
          l1 += (pA[1] + pA[3]) + (pB[1] + pB[3]);
          // P^T as the B operand: transpose the (tok x head) halves
          const uint32_t ba0 = movm_t(pack_bf16x2(pA[0], pA[1]));
          const uint32_t ba1 = movm_t(pack_bf16x2(pA[2], pA[3]));
          const uint32_t bb0 = movm_t(pack_bf16x2(pB[0], pB[1]));
          const uint32_t bb1 = movm_t(pack_bf16x2(pB[2], pB[3]));
          // O^T[128 d][8 heads] += V_A^T P_A^T + V_B^T P_B^T
          const uint32_t vA = kA + TILE, vB = kB + TILE;
#pragma unroll
          for (int t = 0; t < 8; t++) {
            uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
            ldsm_x4_t(vA + vofs[t], a0, a1, a2, a3);
            ldsm_x4_t(vB + vofs[t], b0, b1, b2, b3);
            mma_bf16_16816(o[t], a0, a1, a2, a3, ba0, ba1);
            mma_bf16_16816(o[t], b0, b1, b2, b3, bb0, bb1);
          }
        }
        __syncwarp();
        produce(i + STAGES);
        if (two) produce(i + 1 + STAGES);
        __syncwarp();
        i += step;
      }
    }


    // ----- finish the segment: this warp's share (natural-log m)
    float L0 = l0, L1 = l1;
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      L0 += __shfl_xor_sync(0xffffffffu, L0, off);
      L1 += __shfl_xor_sync(0xffffffffu, L1, off);
    }
    const int n0 = 2 * qid, n1 = 2 * qid + 1;  // head columns of this lane
    float mo0 = m0 * LN2, mo1 = m1 * LN2;
    if constexpr (PARTIAL) {
      // Re-base (l, o) from the lazily moved running max to the true maximum
      // of the range, so that m is the maximum score as the triple promises.
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, off));
        tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, off));
      }
      const float f0 = tm0 == -INFINITY ? 0.f : ex2(m0 - tm0);
      const float f1 = tm1 == -INFINITY ? 0.f : ex2(m1 - tm1);
      L0 *= f0; L1 *= f1;
#pragma unroll
      for (int t = 0; t < 8; t++) { o[t][0] *= f0; o[t][2] *= f0; o[t][1] *= f1; o[t][3] *= f1; }
      mo0 = tm0 * LN2; mo1 = tm1 * LN2;
    }
    if (L0 == 0.f) mo0 = -INFINITY;  // no valid token: an empty partial
    if (L1 == 0.f) mo1 = -INFINITY;
    const int cidx = 2 + cb * Hkv + ckvh;  // this segment's merge counter
    const int ca = owner_unit(seg_S, uper, urem), cz = owner_unit(seg_E - 1, uper, urem);
    const int nc = cz - ca + 1;
    // slot of contributor ca + k: its range's first segment (0) or last (1)
    auto slot_of = [&](int k) -> const Partial* {
      return a.partials + 2 * (ca + k) + ((k == 0 && unit_start(ca, uper, urem) < seg_S) ? 1 : 0);
    };

    if (!grouped) {
      // ---- per-warp split: the segment's blocks of this range are all in registers
      if (whole && PARTIAL) {
        const int64_t row = (int64_t)cb * a.H + head0;
        if (quad == 0) {
          if (n0 < G) { a.m_out[row + n0] = mo0; a.l_out[row + n0] = L0; }
          if (n1 < G) { a.m_out[row + n1] = mo1; a.l_out[row + n1] = L1; }
        }
        float* ob = a.o_out + row * D;
#pragma unroll
        for (int t = 0; t < 8; t++) {
          const int d0 = 16 * t + quad;
          if (n0 < G) { ob[n0 * D + d0] = o[t][0]; ob[n0 * D + d0 + 8] = o[t][2]; }
          if (n1 < G) { ob[n1 * D + d0] = o[t][1]; ob[n1 * D + d0 + 8] = o[t][3]; }
        }
      } else if (whole) {
        const float i0 = L0 > 0.f ? 1.f / L0 : 0.f, i1 = L1 > 0.f ? 1.f / L1 : 0.f;
        __nv_bfloat16* ob = a.out + ((int64_t)cb * a.H + head0) * D;
#pragma unroll
        for (int t = 0; t < 8; t++) {
          const int d0 = 16 * t + quad;
          if (n0 < G) {
            ob[n0 * D + d0] = __float2bfloat16_rn(o[t][0] * i0);
            ob[n0 * D + d0 + 8] = __float2bfloat16_rn(o[t][2] * i0);
          }
          if (n1 < G) {
            ob[n1 * D + d0] = __float2bfloat16_rn(o[t][1] * i1);
            ob[n1 * D + d0 + 8] = __float2bfloat16_rn(o[t][3] * i1);
          }
        }
      } else {
        Partial* pp = a.partials + 2 * unit + e_slot;
        if (quad == 0) {
          if (n0 < G) { pp->m[n0] = mo0; pp->l[n0] = L0; }
          if (n1 < G) { pp->m[n1] = mo1; pp->l[n1] = L1; }
        }
#pragma unroll
        for (int t = 0; t < 8; t++) {
          const int d0 = 16 * t + quad;
          if (n0 < G) { pp->o[n0][d0] = o[t][0]; pp->o[n0][d0 + 8] = o[t][2]; }
          if (n1 < G) { pp->o[n1][d0] = o[t][1]; pp->o[n1][d0 + 8] = o[t][3]; }
        }
        __threadfence();  // the partial before the count
        __syncwarp();
        int old = 0;
        if (lane == 0) old = atomicAdd(&a.counters[cidx], 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == nc - 1) {  // the last contributor merges
          __threadfence();
          merge_units_all<PARTIAL>(a, (int64_t)cb * a.H + head0, G, nc, lane, slot_of);
          if (lane == 0) a.counters[cidx] = 0;
        }
      }
    } else {
      // ---- CTA split: stage the warps' shares, combine them (warp w: heads w, w + WARPS, ...)
      WarpPart& wp = wpart[warp];
      if (quad == 0) {
        if (n0 < G) { wp.m[n0] = mo0; wp.l[n0] = L0; }
        if (n1 < G) { wp.m[n1] = mo1; wp.l[n1] = L1; }
      }
      if (L0 > 0.f || L1 > 0.f) {
#pragma unroll
        for (int t = 0; t < 8; t++) {
          const int d0 = 16 * t + quad;
          if (n0 < G) { wp.o[n0][d0] = o[t][0]; wp.o[n0][d0 + 8] = o[t][2]; }
          if (n1 < G) { wp.o[n1][d0] = o[t][1]; wp.o[n1][d0 + 8] = o[t][3]; }
        }
      }
      cta_bar<WARPS>();
      Partial* cpart = a.partials + 2 * unit + e_slot;
      for (int n = warp; n < G; n += WARPS) {
        float mw[WARPS], M = -INFINITY;
#pragma unroll
        for (int w = 0; w < WARPS; w++) { mw[w] = wpart[w].m[n]; M = fmaxf(M, mw[w]); }
        float den = 0.f;
        float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < WARPS; w++) {
          if (mw[w] == -INFINITY) continue;  // uniform over the warp
          const float wt = __expf(mw[w] - M);
          den += wt * wpart[w].l[n];
          const float4 x = reinterpret_cast<const float4*>(wpart[w].o[n])[lane];
          num.x += wt * x.x; num.y += wt * x.y; num.z += wt * x.z; num.w += wt * x.w;
        }
        if (whole) {
          emit_merged<PARTIAL>(a, (int64_t)cb * a.H + head0 + n, lane, M, den, num);
        } else {
          if (lane == 0) { cpart->m[n] = M; cpart->l[n] = den; }
          reinterpret_cast<float4*>(cpart->o[n])[lane] = num;
        }
      }
      if (!whole) __threadfence();  // this CTA's partial before its count
      cta_bar<WARPS>();             // the staged shares may be overwritten from here on
      if (!whole) {
        // the last CTA to finish a split segment merges the CTAs' partials
        if (tid == 0) s_last = atomicAdd(&a.counters[cidx], 1) == nc - 1;
        cta_bar<WARPS>();
        if (s_last) {
          __threadfence();
          for (int n = warp; n < G; n += WARPS)
            merge_units<PARTIAL>(a, (int64_t)cb * a.H + head0 + n, n, nc, lane, slot_of);
          if (tid == 0) a.counters[cidx] = 0;
        }
      }
    }

    // advance to the next non-empty segment of the unit's range
    if (seg_E >= u1) break;
    if (++ckvh == Hkv) {
      ckvh = 0;
      do { cb++; } while (cb < B && prefix[cb + 1] == prefix[cb]);
    }
  }

  if (timed_out) {
    // Drain the loads this warp still has in flight (bounded) before exit.
    for (int k = i_fail; k < p_hi; k++) {
      const int slot = k % STAGES;
      if (!mbar_wait_warp(smem_u32(&wbars[slot]), (uint32_t)((k / STAGES) & 1), a.status)) break;
    }
  }
}

// ------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Warps per CTA (one CTA per SM) and ring depth per warp. Measured on B200
// (C2 step): one consumer warp per SM sub-partition is fastest -- 4 warps
// reach 86 % of the copy bandwidth (4, 5 or 6 stages alike), 8 warps x 3
// stages only 72 %, 3 warps 74 %, 2 warps 52 %. The partial form keeps the
// per-sequence table offsets in shared memory too and runs 5 stages.
#ifndef ZL_DECODE_WARPS
#define ZL_DECODE_WARPS 4
#endif
#ifndef ZL_DECODE_STAGES
#define ZL_DECODE_STAGES 6
#endif
constexpr int kWarps = ZL_DECODE_WARPS;
constexpr int kStages = ZL_DECODE_STAGES;
constexpr int kStagesPartial = kStages - 1;
static_assert(Smem<kWarps, kStages, false>::kTotal <= 232448, "shared memory of the normalised form");
static_assert(Smem<kWarps, kStagesPartial, true>::kTotal <= 232448, "shared memory of the partial form");

// One CTA per SM. With pdl the launch may begin while the previous kernel on
// the stream still runs (programmatic stream serialization); the kernel's
// griddep_wait keeps every dependent access in stream order.
template <typename Kern>
cudaError_t launch_decode(Kern kern, int grid, int smem, cudaStream_t st, const DecodeArgs& args,
                          const CUtensorMap& tk, const CUtensorMap& tv, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args, tk, tv);
}

// Flat work items (sequence, kv head, block) are indexed in 32 bits.
inline bool flat_index_fits(int B, int max_blocks, int Hkv) {
  return (int64_t)B * max_blocks * Hkv < (1ll << 31);
}

}  // namespace

namespace zl {

// 2-D bf16 tensor map over `rows` rows of `cols` elements (row pitch
// `pitch_bytes`), box [box_rows][box_cols], 128-byte swizzle.
zl_status make_tmap_bf16(CUtensorMap* map, const void* ptr, uint64_t cols, uint64_t rows,
                         uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(ZL_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(ZL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for %llu x %llu", (int)r,
                     (unsigned long long)rows, (unsigned long long)cols);
  return ZL_OK;
}

zl_status launch_decode_bf16_fast(zl_ctx* ctx, const void* q, const void* k_pool, const void* v_pool,
                                  const int32_t* block_tables, const int32_t* seq_lens,
                                  const int32_t* tok_begin, void* out, float* m_out, float* l_out,
                                  float* o_out, int B, int H, int Hkv, int d, int bs, int max_blocks,
                                  int64_t num_blocks, float scale, zl_gqa_map map, int num_splits,
                                  cudaStream_t st) {
  (void)num_splits;
  const bool partial = o_out != nullptr;
  if (d != D || bs != BS || Hkv <= 0 || H % Hkv != 0 || H / Hkv > MAX_G || B > MAX_B ||
      map != ZL_GQA_GROUPED && H != Hkv)
    return ZL_ERR_UNSUPPORTED;
  const uint64_t rows = (uint64_t)num_blocks * Hkv * BS;
  if (rows == 0 || rows >= (1ull << 31) || !flat_index_fits(B, max_blocks, Hkv)) return ZL_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool) |
       reinterpret_cast<uintptr_t>(partial ? (void*)o_out : out)) & 15)
    return ZL_ERR_UNSUPPORTED;
  if (B == 0) return ZL_OK;

  CUtensorMap tk, tv;
  zl_status s = make_tmap_bf16(&tk, k_pool, D, rows, D * 2, 64, BS);
  if (s != ZL_OK) return s;
  s = make_tmap_bf16(&tv, v_pool, D, rows, D * 2, 64, BS);
  if (s != ZL_OK) return s;

  const int grid = ctx->num_sms;
  s = ensure_workspace(ctx, sizeof(Partial) * 2 * grid * kWarps);
  if (s != ZL_OK) return s;
  s = ensure_counters(ctx, sizeof(int) * (2 + (size_t)B * Hkv));
  if (s != ZL_OK) return s;

  DecodeArgs args;
  args.q = (const __nv_bfloat16*)q;
  args.block_tables = block_tables;
  args.seq_lens = seq_lens;
  args.tok_begin = tok_begin;
  args.out = (__nv_bfloat16*)out;
  args.m_out = m_out;
  args.l_out = l_out;
  args.o_out = o_out;
  args.partials = (Partial*)ctx->workspace;
  args.counters = (int*)ctx->counters;
  args.status = ctx->d_status;
  args.B = B; args.H = H; args.Hkv = Hkv; args.G = H / Hkv; args.max_blocks = max_blocks;
  args.num_blocks = num_blocks;
  args.scale_log2 = scale * LOG2E;
  args.inputs_ahead = (ctx->flags & ZL_CTX_INPUTS_AHEAD) ? 1 : 0;

  // the shared-memory limit is a per-device attribute of each function
  auto set_smem = [&](auto kern, int bytes, std::atomic<uint64_t>& done) -> cudaError_t {
    if (ctx->device < 64 && !(done.load() & (1ull << ctx->device))) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      if (e != cudaSuccess) return e;
      done.fetch_or(1ull << ctx->device);
    }
    return cudaSuccess;
  };
  if (partial) {
    using SM = Smem<kWarps, kStagesPartial, true>;
    auto kern = paged_decode_bf16_kernel<kWarps, kStagesPartial, true>;
    static std::atomic<uint64_t> attr_set{0};
    ZL_CUDA_TRY(set_smem(kern, SM::kTotal, attr_set));
    ZL_CUDA_TRY(launch_decode(kern, grid, SM::kTotal, st, args, tk, tv, true));
  } else {
    using SM = Smem<kWarps, kStages, false>;
    auto kern = paged_decode_bf16_kernel<kWarps, kStages, false>;
    static std::atomic<uint64_t> attr_set{0};
    ZL_CUDA_TRY(set_smem(kern, SM::kTotal, attr_set));
    ZL_CUDA_TRY(launch_decode(kern, grid, SM::kTotal, st, args, tk, tv, true));
  }
  ZL_LAUNCH_CHECK(ctx);
  return ZL_OK;
}

}  // namespace zl

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// zl_paged_decode keeps its split-KV partials and merge counters in a context
// workspace that it grows with cudaMalloc on first use and whenever a batch
// needs more. Some callers cannot allow that: a serving engine that hands
// (nearly) all HBM to its KV-cache pool at start-up has nothing left for an
// on-demand allocation, and a step loop that must not stall cannot accept
// the device-wide synchronisation cudaMalloc/cudaFree imply. For them,
// zl_paged_decode_noalloc runs the same kernel with its scratch in the
// file-scope array below, which is part of the loaded module: every GPU that
// loads this library holds it (about 5.4 MB) until the process exits.
//
// Limits: bf16, head_dim 128, block_size 16, grouped GQA with at most 8
// query heads per kv head, num_seqs <= 4096, num_seqs * num_kv_heads <=
// kNoAllocMaxSegments. Larger requests are rejected with an error.
// All calls share the array: two calls whose kernels overlap on the GPU (on
// different streams, or from different host threads without ordering) race
// on it and give wrong results. Calls ordered on one stream are safe; each
// call clears the merge counters it uses before its kernel runs.
// Device-side errors go to the caller's status word, which is required: the
// call itself returns ZL_OK once the kernel is queued.
namespace {

constexpr int kNoAllocMaxCtas = 160;            // >= 148 SMs of a B200
constexpr int kNoAllocMaxSegments = 16384;      // (sequence, kv head) pairs per call
struct NoAllocScratch {
  Partial partials[2 * kNoAllocMaxCtas * kWarps];
  int counters[2 + kNoAllocMaxSegments];  // grid-barrier words, then one per (sequence, kv head)
};
static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

constexpr int kMaxDevices = 64;
struct NoAllocDevice {
  NoAllocScratch* scratch = nullptr;  // device address of g_noalloc_scratch when last resolved
  int num_sms = 0;
};
NoAllocDevice g_noalloc_dev[kMaxDevices];
std::mutex g_noalloc_mu;

// Every call, with the device current: resolve the array's device address
// (the host-side symbol is only a stand-in and must never be handed to a
// kernel; the lookup is cheap and allocates nothing). When the address is new
// -- the first call on the device, or the module was loaded again after a
// device reset -- also read the SM count and raise the kernel's dynamic
// shared-memory limit, which a reset drops as well.
zl_status noalloc_setup(int dev, NoAllocDevice** out) {
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  NoAllocDevice& nd = g_noalloc_dev[dev];
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess)
    return zl::set_error(ZL_ERR_CUDA, "paged_decode_noalloc: cudaGetSymbolAddress failed: %s",
                         cudaGetErrorString(e));
  if (nd.scratch != p) {
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess)
      return zl::set_error(ZL_ERR_CUDA, "paged_decode_noalloc: SM count: %s", cudaGetErrorString(e));
    using SM = Smem<kWarps, kStages, false>;
    e = cudaFuncSetAttribute(paged_decode_bf16_kernel<kWarps, kStages, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SM::kTotal);
    if (e != cudaSuccess)
      return zl::set_error(ZL_ERR_CUDA, "paged_decode_noalloc: shared-memory limit: %s",
                           cudaGetErrorString(e));
    nd.num_sms = sms;
    nd.scratch = reinterpret_cast<NoAllocScratch*>(p);
  }
  *out = &nd;
  return ZL_OK;
}

}  // namespace

extern "C" zl_status zl_paged_decode_noalloc(const void* q, const void* k_pool, const void* v_pool,
                                             const int32_t* block_tables, const int32_t* seq_lens,
                                             void* out, int* status, int num_seqs, int num_heads,
                                             int num_kv_heads, int head_dim, int block_size,
                                             int max_blocks_per_seq, int64_t num_blocks,
                                             float scale, zl_stream stream) {
  using namespace zl;
  if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_blocks_per_seq < 0 || num_blocks < 0)
    return set_error(ZL_ERR_INVALID_ARG, "paged_decode_noalloc: bad sizes");
  if (head_dim != D || block_size != BS || num_heads % num_kv_heads != 0 ||
      num_heads / num_kv_heads > MAX_G)
    return set_error(ZL_ERR_UNSUPPORTED,
                     "paged_decode_noalloc: needs head_dim 128, block_size 16 and at most %d query "
                     "heads per kv head (got d=%d bs=%d H=%d Hkv=%d)",
                     MAX_G, head_dim, block_size, num_heads, num_kv_heads);
  if (num_seqs > MAX_B || (int64_t)num_seqs * num_kv_heads > kNoAllocMaxSegments)
    return set_error(ZL_ERR_INVALID_ARG,
                     "paged_decode_noalloc: %d sequences x %d kv heads exceed the static scratch "
                     "(at most %d sequences and %d sequence-kv-head pairs)",
                     num_seqs, num_kv_heads, MAX_B, kNoAllocMaxSegments);
  const uint64_t rows = (uint64_t)num_blocks * num_kv_heads * BS;
  if (rows >= (1ull << 31))
    return set_error(ZL_ERR_INVALID_ARG, "paged_decode_noalloc: pool of %lld blocks is too large",
                     (long long)num_blocks);
  if (!flat_index_fits(num_seqs, max_blocks_per_seq, num_kv_heads))
    return set_error(ZL_ERR_INVALID_ARG, "paged_decode_noalloc: num_seqs x max_blocks_per_seq x num_kv_heads "
                     "must stay below 2^31");
  if (!status)
    return set_error(ZL_ERR_INVALID_ARG,
                     "paged_decode_noalloc: a device status word is required (device-side errors "
                     "are reported only there)");
  if (num_seqs == 0) return ZL_OK;
  if (!q || !k_pool || !v_pool || !block_tables || !seq_lens || !out || rows == 0)
    return set_error(ZL_ERR_INVALID_ARG, "paged_decode_noalloc: null pointer or empty pool");
  if ((reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool) |
       reinterpret_cast<uintptr_t>(out)) & 15)
    return set_error(ZL_ERR_INVALID_ARG, "paged_decode_noalloc: pools and out must be 16-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(ZL_ERR_CUDA, "paged_decode_noalloc: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(ZL_ERR_UNSUPPORTED, "device ordinal %d", dev);
  NoAllocDevice* nd = nullptr;
  zl_status s = noalloc_setup(dev, &nd);
  if (s != ZL_OK) return s;

  CUtensorMap tk, tv;
  if ((s = make_tmap_bf16(&tk, k_pool, D, rows, D * 2, 64, BS)) != ZL_OK) return s;
  if ((s = make_tmap_bf16(&tv, v_pool, D, rows, D * 2, 64, BS)) != ZL_OK) return s;

  cudaStream_t st = S(stream);
  NoAllocScratch* scr = nd->scratch;
  // The grid-barrier words and the merge counters of this call's (sequence,
  // kv head) pairs must start at zero; clearing them per call also recovers
  // from a call whose kernel gave up part-way.
  e = cudaMemsetAsync(scr->counters, 0, sizeof(int) * (2 + (size_t)num_seqs * num_kv_heads), st);
  if (e != cudaSuccess) return set_error(ZL_ERR_CUDA, "paged_decode_noalloc: counter clear: %s", cudaGetErrorString(e));

  DecodeArgs args;
  args.q = (const __nv_bfloat16*)q;
  args.block_tables = block_tables;
  args.seq_lens = seq_lens;
  args.tok_begin = nullptr;
  args.out = (__nv_bfloat16*)out;
  args.m_out = args.l_out = args.o_out = nullptr;
  args.partials = scr->partials;
  args.counters = scr->counters;
  args.status = status;
  args.B = num_seqs; args.H = num_heads; args.Hkv = num_kv_heads; args.G = num_heads / num_kv_heads;
  args.max_blocks = max_blocks_per_seq;
  args.num_blocks = num_blocks;
  args.scale_log2 = resolve_scale(scale, D) * LOG2E;
  args.inputs_ahead = 0;
  const int grid = nd->num_sms < kNoAllocMaxCtas ? nd->num_sms : kNoAllocMaxCtas;
  using SM = Smem<kWarps, kStages, false>;
  e = launch_decode(paged_decode_bf16_kernel<kWarps, kStages, false>, grid, SM::kTotal, st, args, tk, tv,
                    false);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(ZL_ERR_CUDA, "paged_decode_noalloc: launch: %s", cudaGetErrorString(e));
  return ZL_OK;
}
