// prefill_tc.cu -- variable-length causal prefill attention on the sm_100a
// tensor cores (tcgen05 + TMEM, fed by TMA), bf16 in, fp32 accumulate.
//
// Replaces tiled_attention_kernel (src/attention/kernels/attention.cu:9-187
// of the reference: scalar fp32 FMAs over shared memory, one sequence in
// [H][L][d]) for packed varlen input q [T][H][128], k/v [T][Hkv][128].
//
// A work item is a 128-row query tile of one sequence for TWO query heads of
// the same kv group, so every K/V tile it loads feeds two score tiles. The
// kernel is persistent (one CTA per SM); items are taken heaviest first from a
// device counter, and the next item's Q load and first score products overlap
// the current item's last tiles and epilogue:
//   warp 0      work fetch + TMA producer: Q tiles once per item, K/V tiles
//               through a 2-stage ring
//   warp 1      MMA issuer (one thread) + TMEM owner (alloc/dealloc 512 cols)
//   warps 4-7   softmax warpgroup for head 0, one thread per query row
//   warps 8-11  softmax warpgroup for head 1
// TMEM columns: S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512); the bf16
// probabilities P overwrite the first 64 columns of their S tile and feed
// O += P V straight from TMEM. The MMA warp interleaves the two heads
// (PV0(j), S0(j+1), PV1(j), S1(j+1)) so one warpgroup's softmax overlaps the
// other's matrix products. Causal tiles past the diagonal are never loaded.
// The softmax is bound by instruction issue as much as by the MUFU unit, so
// its arithmetic runs on packed fp32 pairs (FFMA2/FADD2, three-input max) and
// one exponential in eight runs on the FMA pipe instead of MUFU.
// Every mbarrier wait is bounded (status word + unwind instead of a hang).
#include "zl_internal.h"
#include "zl_ptx.cuh"

namespace zl {
zl_status make_tmap_bf16(CUtensorMap* map, const void* ptr, uint64_t cols, uint64_t rows,
                         uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows);
}

namespace {

using namespace zl::ptx;

constexpr int D = 128;
constexpr int BM = 128;                 // query rows per tile
constexpr int BN = 128;                 // keys per tile
constexpr int NQ = 2;                   // query heads per CTA
constexpr int TILE = BM * D * 2;        // 32 KB (two 16 KB swizzled boxes)
constexpr int HALF = TILE / 2;
constexpr int THREADS = 384;
constexpr float LOG2E = 1.4426950408889634f;

// Per item: Q_FULL / Q_EMPTY (the item's Q tiles loaded / its last score
// products done, so the next item's Q may land), O_FINAL (the item's last
// P V done), O_EMPTY (the epilogue has read O: the next item's first P V may
// overwrite it). Per tile (running count across items): K/V ring, S_FULL,
// P_READY. IT_FULL / IT_EMPTY: a 2-slot ring of fetched item ids.
enum Bar { Q_FULL = 0, Q_EMPTY = 1, K_FULL = 2, K_EMPTY = 4, V_FULL = 6, V_EMPTY = 8, S_FULL = 10,
           P_READY = 12, O_FINAL = 14, O_EMPTY = 16, IT_FULL = 18, IT_EMPTY = 20, NUM_BARS = 22 };
constexpr int IT_READERS = 1 + 8;  // the MMA thread and one lane of each softmax warp

struct Smem {
  static constexpr int kQ = 0;                      // NQ tiles
  static constexpr int kK = kQ + NQ * TILE;         // 2 stages
  static constexpr int kV = kK + 2 * TILE;          // 2 stages
  static constexpr int kBars = kV + 2 * TILE;
  static constexpr int kItems = kBars + NUM_BARS * 8;  // 2 fetched item ids
  static constexpr int kTmem = kItems + 8;
  static constexpr int kTotal = 1024 + kTmem + 16;
};

struct PrefillArgs {
  const int32_t* cu_seqlens;
  __nv_bfloat16* out;  // [T][H][D]
  int* status;
  int* work;             // [0] next item, [1] CTAs finished; zero between launches
  int64_t total_tokens;  // rows of q / k / v / out: every sequence must end at or before it
  int H, Hkv, G, num_seqs;
  int hp_count, max_tiles, total_items;
  float scale_log2;
  int causal;
};

// Item idx -> (sequence, head pair, query tile); items run heaviest (latest
// tile) first. nkv: K/V tiles to visit; 0 = the tile is past the sequence;
// -1 = cu_seqlens is malformed for this sequence.
struct Item {
  int s, hp, t, start, L, nkv;
};
__device__ __forceinline__ Item decode_item(const PrefillArgs& a, int idx) {
  Item it;
  const int xy = a.num_seqs * a.hp_count;
  const int y = idx / xy, x = idx - y * xy;
  it.t = a.max_tiles - 1 - y;
  it.s = x / a.hp_count;
  it.hp = x - it.s * a.hp_count;
  it.start = a.cu_seqlens[it.s];
  const int end = a.cu_seqlens[it.s + 1];
  it.L = end - it.start;
  // cu_seqlens comes from device memory: a sequence outside [0, total_tokens]
  // or running backwards is reported and skipped, so no load or store leaves
  // the caller's buffers. A sequence longer than the launch's max_seq_len
  // (rows no tile covers) is reported and skipped too.
  if (it.start < 0 || end < it.start || (int64_t)end > a.total_tokens ||
      (int64_t)it.L > (int64_t)BM * a.max_tiles)
    it.nkv = -1;
  else if (BM * it.t >= it.L)
    it.nkv = 0;
  else
    it.nkv = a.causal ? it.t + 1 : (it.L + BN - 1) / BN;
  return it;
}

constexpr uint32_t IDESC_S = idesc_bf16(BM, BN, false, false);
constexpr uint32_t IDESC_PV = idesc_bf16(BM, D, false, true);

// K-major, 128-byte swizzle operand (Q or K tile): k-step kk covers 16 of the
// 128 head dims; dims 0-63 live in the first 16 KB box, 64-127 in the second.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile, int kk) {
  return sdesc(tile + (kk >> 2) * HALF + (kk & 3) * 32, 16, 1024, 2);
}
// MN-major, 128-byte swizzle B operand (V tile as [keys][dims]): k-step kk
// covers keys 16kk..16kk+15; the two 64-dim boxes are LBO = 16 KB apart.
__device__ __forceinline__ uint64_t desc_v(uint32_t tile, int kk) {
  return sdesc(tile + kk * 2048, HALF, 1024, 2);
}

// 2^x on the FMA and integer pipes, for the share of the softmax exponentials
// taken off the MUFU unit: x = j + f with j = rint(x) (adding 1.5 * 2^23 leaves
// j in the low mantissa bits) and f in [-0.5, 0.5]; 2^f by a cubic fitted to 2^f
// on that interval (reweighted least squares, max relative error 7.5e-5, well
// under the bf16 rounding of P); j is added to the exponent field. x is clamped
// at -125 so the exponent stays normal (2^-125 ~ 2e-38 is zero for every use
// here).
__device__ __forceinline__ float ex2_fma(float x) {
  x = fmaxf(x, -125.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  const float p = fmaf(fmaf(fmaf(0.05517166f, f, 0.24261113f), f, 0.69326097f), f, 0.99992806f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

__global__ void __launch_bounds__(THREADS, 1)
prefill_tc_kernel(const PrefillArgs a, const __grid_constant__ CUtensorMap tmQ,
                  const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sbase = smem_raw + (base - raw);
  auto bar = [&](int i) { return base + Smem::kBars + 8 * i; };
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(sbase + Smem::kTmem);
  volatile int* items = reinterpret_cast<volatile int*>(sbase + Smem::kItems);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NUM_BARS; i++) {
      int count = 1;
      if (i == P_READY || i == P_READY + 1 || i == O_EMPTY || i == O_EMPTY + 1) count = 128;
      if (i == IT_EMPTY || i == IT_EMPTY + 1) count = IT_READERS;
      mbar_init(bar(i), count);
    }
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    __syncwarp();  // tcgen05.alloc/dealloc are warp-collective (.sync.aligned)
    tmem_alloc(base + Smem::kTmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS[2] = {tmem, tmem + 128};
  const uint32_t tO[2] = {tmem + 256, tmem + 384};

  if (warp < 4) {
  if (warp == 0 && lane == 0) {
    // ------------------------------------------------- work fetch + producer
    // Item k goes to slot k & 1 of the item ring; the id past the last item
    // (or once a wait anywhere timed out) tells the other roles to stop.
    int q_it = 0, g = 0;  // items with work, K/V tiles loaded (running counts)
    for (int k = 0;; k++) {
      const int slot = k & 1;
      if (!mbar_wait(bar(IT_EMPTY + slot), ((k >> 1) & 1) ^ 1, a.status)) break;
      const int idx = aborted(a.status) ? a.total_items : atomicAdd(a.work, 1);
      items[slot] = idx < a.total_items ? idx : a.total_items;
      mbar_arrive(bar(IT_FULL + slot));  // release: the id is visible to the waiters
      if (idx >= a.total_items) break;
      const Item it = decode_item(a, idx);
      if (it.nkv < 0) atomicOr(a.status, ZL_DEV_OOB);
      if (it.nkv <= 0) continue;
      const int h0 = it.hp * NQ, kvh = h0 / a.G;
      // the Q buffer is free once the previous item's last score products are done
      if (!mbar_wait(bar(Q_EMPTY), (q_it & 1) ^ 1, a.status)) break;
      const int y0 = it.start + BM * it.t;
      mbar_arrive_expect_tx(bar(Q_FULL), NQ * TILE);
      for (int w = 0; w < NQ; w++) {
        const uint32_t dst = base + Smem::kQ + w * TILE;
        tma_load_2d(dst, &tmQ, (h0 + w) * D, y0, bar(Q_FULL));
        tma_load_2d(dst + HALF, &tmQ, (h0 + w) * D + 64, y0, bar(Q_FULL));
      }
      bool ok = true;
      for (int j = 0; j < it.nkv; j++, g++) {
        const int st = g & 1;
        const uint32_t ph = (g >> 1) & 1;
        const int y = it.start + BN * j;
        if (!(ok = mbar_wait(bar(K_EMPTY + st), ph ^ 1, a.status))) break;
        mbar_arrive_expect_tx(bar(K_FULL + st), TILE);
        tma_load_2d(base + Smem::kK + st * TILE, &tmK, kvh * D, y, bar(K_FULL + st));
        tma_load_2d(base + Smem::kK + st * TILE + HALF, &tmK, kvh * D + 64, y, bar(K_FULL + st));
        if (!(ok = mbar_wait(bar(V_EMPTY + st), ph ^ 1, a.status))) break;
        mbar_arrive_expect_tx(bar(V_FULL + st), TILE);
        tma_load_2d(base + Smem::kV + st * TILE, &tmV, kvh * D, y, bar(V_FULL + st));
        tma_load_2d(base + Smem::kV + st * TILE + HALF, &tmV, kvh * D + 64, y, bar(V_FULL + st));
      }
      if (!ok) break;
      q_it++;
    }
  } else if (warp == 1 && lane == 0) {
    // ----------------------------------------------------------- MMA issuer
    // step-0 descriptors of every operand tile, computed once: each group of
    // eight MMAs is then one asm block (tc_mma_*_k128). The single issuing
    // thread's dependent instruction chain per MMA (descriptor arithmetic,
    // predicate, issue) otherwise sets the rate at which products reach the
    // tensor pipe.
    const uint64_t dq0 = desc_kmajor(base + Smem::kQ, 0), dq1 = desc_kmajor(base + Smem::kQ + TILE, 0);
    const uint64_t dk0 = desc_kmajor(base + Smem::kK, 0), dk1 = desc_kmajor(base + Smem::kK + TILE, 0);
    const uint64_t dv0 = desc_v(base + Smem::kV, 0), dv1 = desc_v(base + Smem::kV + TILE, 0);
    auto issue_s = [&](int w, int st) {
      tc_mma_ss_k128(tS[w], w ? dq1 : dq0, st ? dk1 : dk0, IDESC_S, 0u);
    };
    auto issue_pv = [&](int w, int st, bool acc) {
      tc_mma_ts_k128(tO[w], tS[w], st ? dv1 : dv0, IDESC_PV, acc ? 1u : 0u);
    };
    int q_it = 0, g = 0;  // items with work, tiles (running counts)
    bool ok = true;
    for (int k = 0; ok; k++) {
      const int slot = k & 1;
      if (!(ok = mbar_wait(bar(IT_FULL + slot), (k >> 1) & 1, a.status))) break;
      const int idx = items[slot];
      mbar_arrive(bar(IT_EMPTY + slot));
      if (idx >= a.total_items) break;
      const Item it = decode_item(a, idx);
      if (it.nkv <= 0) continue;
      const int nkv = it.nkv;
      // S(0) of both heads: the S columns are free (this thread issued the
      // previous item's last P V before, and the products complete in order)
      if (!(ok = mbar_wait(bar(Q_FULL), q_it & 1, a.status))) break;
      if (!(ok = mbar_wait(bar(K_FULL + (g & 1)), (g >> 1) & 1, a.status))) break;
      tc_fence_after();
      for (int w = 0; w < NQ; w++) {
        issue_s(w, g & 1);
        tc_commit(bar(S_FULL + w));
      }
      tc_commit(bar(K_EMPTY + (g & 1)));
      if (nkv == 1) tc_commit(bar(Q_EMPTY));  // every score product of this item issued
      for (int j = 0; ok && j < nkv; j++) {
        const int gj = g + j;
        const int st = gj & 1;
        const uint32_t ph = (gj >> 1) & 1;
        const int st1 = (gj + 1) & 1;
        const uint32_t ph1 = ((gj + 1) >> 1) & 1;
        if (!(ok = mbar_wait(bar(V_FULL + st), ph, a.status))) break;
        // The next tile's K usually landed long ago: probed here, while P of
        // head 0 is still being written, a completed K needs no wait between
        // head 0's P V and its next scores.
        bool k_next = j + 1 < nkv && mbar_test(bar(K_FULL + st1), ph1);
        for (int w = 0; w < NQ && ok; w++) {
          if (!(ok = mbar_wait(bar(P_READY + w), gj & 1, a.status))) break;
          // the first P V of an item overwrites O: the previous item's epilogue must have read it
          if (j == 0 && q_it > 0 && !(ok = mbar_wait(bar(O_EMPTY + w), (q_it - 1) & 1, a.status))) break;
          tc_fence_after();
          issue_pv(w, st, j > 0);
          if (w == NQ - 1) tc_commit(bar(V_EMPTY + st));
          if (j + 1 < nkv) {
            if (w == 0 && !k_next && !(ok = mbar_wait(bar(K_FULL + st1), ph1, a.status))) break;
            tc_fence_after();
            issue_s(w, st1);
            tc_commit(bar(S_FULL + w));
            if (w == NQ - 1) {
              tc_commit(bar(K_EMPTY + st1));
              if (j + 2 == nkv) tc_commit(bar(Q_EMPTY));
            }
          } else {
            tc_commit(bar(O_FINAL + w));
          }
        }
      }
      g += nkv;
      q_it++;
    }
  }
  } else {
    // ------------------------------------------------------ softmax + epilogue
    const int w = (warp - 4) >> 2;             // which query head of the pair
    const int r = 32 * (warp & 3) + lane;      // query row in the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const uint32_t tSr = tS[w] + lane_off, tOr = tO[w] + lane_off;
    // The running max only moves when a tile's row max exceeds it by more
    // than 2^8: until then p = 2^(s - m) <= 256 is exact enough in bf16/fp32
    // and the O rescale (a TMEM round trip of 128 columns) is skipped.
    constexpr float kLazy = 8.f;
    const float sc = a.scale_log2;
    bool ok = true;
    int q_it = 0, g = 0;  // items with work, tiles (running counts)
    for (int k = 0; ok; k++) {
    const int slot = k & 1;
    if (!(ok = mbar_wait_warp(bar(IT_FULL + slot), (k >> 1) & 1, a.status))) break;
    const int idx = items[slot];
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(IT_EMPTY + slot));
    if (idx >= a.total_items) break;
    const Item it = decode_item(a, idx);
    if (it.nkv <= 0) continue;
    const int t = it.t, L = it.L, start = it.start, nkv = it.nkv, h0 = it.hp * NQ;
    const int q_row = BM * t + r;              // row index within the sequence
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < nkv; j++) {
      if (!(ok = mbar_wait_warp(bar(S_FULL + w), (g + j) & 1, a.status))) break;
      tc_fence_after();
      // only the last tile of a row range needs a mask (the diagonal when causal)
      const bool edge = (j == nkv - 1) && (a.causal || (L % BN) != 0);
      const int key_lim = edge ? (a.causal ? min(q_row + 1, L) : L) - BN * j : BN;
      uint32_t va[32], vb[32];
      // Speculative single pass (interior tiles after the first): the
      // exponentials are taken against the running max as it stands while the
      // tile's own max is tracked alongside, so the max pass (two TMEM loads
      // and the max chain) leaves the softmax's critical path. The tile is
      // done in two 64-key halves. If a row of the first half beats the
      // running max by more than 2^8, nothing has been stored and the
      // two-pass path below redoes the tile; if only the second half does, the
      // first half's P (already in TMEM) is re-based to the new max in place.
      bool done = false;
      if (j > 0 && !edge) {
        uint32_t pa[16], pb[16];
        float mx8[8];
        uint64_t ls2[4];
        const uint64_t sc2 = f2_pack(sc, sc);
        // exponentials of one half against max mref, P packed into pa / pb
        auto half_exp = [&](float mref) {
          const uint64_t nm2 = f2_pack(-mref, -mref);
#pragma unroll
          for (int u = 0; u < 4; u++) ls2[u] = 0ull;
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const float a0 = __uint_as_float(va[2 * i]), a1 = __uint_as_float(va[2 * i + 1]);
            const float b0 = __uint_as_float(vb[2 * i]), b1 = __uint_as_float(vb[2 * i + 1]);
            const float2 xa = f2_unpack(f2_fma(f2_pack(a0, a1), sc2, nm2));
            const float2 xb = f2_unpack(f2_fma(f2_pack(b0, b1), sc2, nm2));
            const float p0 = ex2(xa.x), p1 = ex2(xa.y), p2 = ex2(xb.x);
            const float p3 = (i & 1) ? ex2_fma(xb.y) : ex2(xb.y);
            ls2[(2 * i) & 3] = f2_add(ls2[(2 * i) & 3], f2_pack(p0, p1));
            ls2[(2 * i + 1) & 3] = f2_add(ls2[(2 * i + 1) & 3], f2_pack(p2, p3));
            pa[i] = pack_bf16x2(p0, p1);
            pb[i] = pack_bf16x2(p2, p3);
          }
          float ls8[8];
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const float2 v = f2_unpack(ls2[u]);
            ls8[2 * u] = v.x;
            ls8[2 * u + 1] = v.y;
          }
          return ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
        };
        auto half_max = [&]() {
#pragma unroll
          for (int u = 0; u < 8; u++) mx8[u] = -INFINITY;
#pragma unroll
          for (int i = 0; i < 32; i++)
            mx8[i & 7] = max3(mx8[i & 7], __uint_as_float(va[i]), __uint_as_float(vb[i]));
          return fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                       fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) * sc;
        };
        tmem_ld32(tSr, va);
        tmem_ld32(tSr + 32, vb);
        tc_wait_ld();
        const float ls_a = half_exp(m);
        const float mt_a = half_max();
        if (!__any_sync(0xffffffffu, mt_a > m + kLazy)) {
          tmem_st16(tSr, pa);          // P of keys 0-63 over S columns 0-31
          tmem_st16(tSr + 16, pb);
          tmem_ld32(tSr + 64, va);     // S of keys 64-127 (columns 64-127, untouched)
          tmem_ld32(tSr + 96, vb);
          tc_wait_ld();
          float ls_b = half_exp(m);
          const float mt_b = half_max();
          float ls_prev = l + ls_a;
          if (__any_sync(0xffffffffu, mt_b > m + kLazy)) {
            // rare: the second half moved the max; re-base to it (S of the
            // second half is reloaded afterwards: its registers are reused)
            const float m_new = fmaxf(m, mt_b);
            const float alpha = ex2(m - m_new);  // 1 for rows whose max did not move
            uint32_t vp[32];
            tmem_ld32(tSr, vp);                  // the first half's P, bf16 pairs
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; i++) {
              const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vp[i]));
              vp[i] = pack_bf16x2(f.x * alpha, f.y * alpha);
            }
            tmem_st32(tSr, vp);
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {     // O of this row by alpha
              tmem_ld32(tOr + 64 * hh, va);
              tmem_ld32(tOr + 64 * hh + 32, vb);
              tc_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; i++) {
                va[i] = __float_as_uint(__uint_as_float(va[i]) * alpha);
                vb[i] = __float_as_uint(__uint_as_float(vb[i]) * alpha);
              }
              tmem_st32(tOr + 64 * hh, va);
              tmem_st32(tOr + 64 * hh + 32, vb);
            }
            ls_prev *= alpha;
            m = m_new;
            tmem_ld32(tSr + 64, va);
            tmem_ld32(tSr + 96, vb);
            tc_wait_ld();
            ls_b = half_exp(m);
          }
          tmem_st16(tSr + 32, pa);     // P of keys 64-127 over S columns 32-63
          tmem_st16(tSr + 48, pb);
          l = ls_prev + ls_b;
          done = true;
        }
      }
      if (!done) {
      // 8 independent max accumulators: a 128-long dependent fmax chain would
      // dominate the row's latency
      float mx8[8];
#pragma unroll
      for (int u = 0; u < 8; u++) mx8[u] = -INFINITY;
#pragma unroll
      for (int hh = 0; hh < 2; hh++) {  // two 32-column chunks per TMEM wait
        tmem_ld32(tSr + 64 * hh, va);
        tmem_ld32(tSr + 64 * hh + 32, vb);
        tc_wait_ld();
        if (edge) {
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const float xa = (64 * hh + i < key_lim) ? __uint_as_float(va[i]) : -INFINITY;
            const float xb = (64 * hh + 32 + i < key_lim) ? __uint_as_float(vb[i]) : -INFINITY;
            mx8[i & 7] = fmaxf(mx8[i & 7], fmaxf(xa, xb));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; i++)
            mx8[i & 7] = max3(mx8[i & 7], __uint_as_float(va[i]), __uint_as_float(vb[i]));
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float m_tile = mx * sc;
      const bool grow = m_tile > m + kLazy;
      const bool any_grow = __any_sync(0xffffffffu, grow);
      const float m_new = grow ? fmaxf(m, m_tile) : m;
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = (m == -INFINITY) ? 0.f : ex2(m - m_use);
      // four pair accumulators for the row sum; x = s * scale - m as fp32 pairs
      uint64_t ls2[4];
#pragma unroll
      for (int u = 0; u < 4; u++) ls2[u] = 0ull;
      const uint64_t sc2 = f2_pack(sc, sc), nm2 = f2_pack(-m_use, -m_use);
#pragma unroll
      for (int hh = 0; hh < 2; hh++) {
        tmem_ld32(tSr + 64 * hh, va);
        tmem_ld32(tSr + 64 * hh + 32, vb);
        tc_wait_ld();
        uint32_t pa[16], pb[16];
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int k0 = 64 * hh + 2 * i, k1 = k0 + 32;
          const float2 xa = f2_unpack(f2_fma(f2_pack(__uint_as_float(va[2 * i]), __uint_as_float(va[2 * i + 1])), sc2, nm2));
          const float2 xb = f2_unpack(f2_fma(f2_pack(__uint_as_float(vb[2 * i]), __uint_as_float(vb[2 * i + 1])), sc2, nm2));
          float p0 = ex2(xa.x), p1 = ex2(xa.y), p2 = ex2(xb.x);
          float p3 = (i & 1) ? ex2_fma(xb.y) : ex2(xb.y);
          if (edge) {  // masked keys: 0 (the FMA form would give 2^-125 for -inf)
            p0 = k0 < key_lim ? p0 : 0.f;
            p1 = k0 + 1 < key_lim ? p1 : 0.f;
            p2 = k1 < key_lim ? p2 : 0.f;
            p3 = k1 + 1 < key_lim ? p3 : 0.f;
          }
          ls2[(2 * i) & 3] = f2_add(ls2[(2 * i) & 3], f2_pack(p0, p1));
          ls2[(2 * i + 1) & 3] = f2_add(ls2[(2 * i + 1) & 3], f2_pack(p2, p3));
          pa[i] = pack_bf16x2(p0, p1);
          pb[i] = pack_bf16x2(p2, p3);
        }
        // P over the first 64 columns of S: chunk c goes to columns [16c, 16c+16),
        // all below the S columns still to be read
        tmem_st16(tSr + 32 * hh, pa);
        tmem_st16(tSr + 32 * hh + 16, pb);
      }
      float ls8[8];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float2 v = f2_unpack(ls2[u]);
        ls8[2 * u] = v.x;
        ls8[2 * u + 1] = v.y;
      }
      const float lsum = ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
      l = l * alpha + lsum;
      // tcgen05.ld/st are warp-collective: the rescale branch is taken by the
      // whole warp (rows whose max did not move multiply by alpha == 1).
      if (j > 0 && any_grow) {
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
          tmem_ld32(tOr + 64 * hh, va);
          tmem_ld32(tOr + 64 * hh + 32, vb);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; i++) {
            va[i] = __float_as_uint(__uint_as_float(va[i]) * alpha);
            vb[i] = __float_as_uint(__uint_as_float(vb[i]) * alpha);
          }
          tmem_st32(tOr + 64 * hh, va);
          tmem_st32(tOr + 64 * hh + 32, vb);
        }
      }
      m = m_new;
      }  // two-pass path
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(bar(P_READY + w));
    }
    if (!ok) break;
    if (!(ok = mbar_wait_warp(bar(O_FINAL + w), q_it & 1, a.status))) break;
    {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool row_ok = q_row < L;
      uint4* dst = reinterpret_cast<uint4*>(a.out + ((int64_t)(start + q_row) * a.H + h0 + w) * D);
#pragma unroll
      for (int c = 0; c < 4; c++) {
        uint32_t v[32];
        tmem_ld32(tOr + 32 * c, v);
        tc_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; i++)
          pk[i] = pack_bf16x2(__uint_as_float(v[2 * i]) * inv, __uint_as_float(v[2 * i + 1]) * inv);
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 4; i++)
            dst[4 * c + i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
    }
    // O has been read: the next item's first P V may overwrite it
    tc_fence_before();
    mbar_arrive(bar(O_EMPTY + w));
    g += nkv;
    q_it++;
    }  // item loop
  }
  __syncwarp();  // lanes of warps 0 and 1 arrive from different roles
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // lane 0 arrives here from the MMA role, lanes 1-31 from the barrier:
    // reconverge the warp before the warp-collective dealloc.
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0) {
    // Every CTA has stopped taking items once it gets here; the last one to
    // finish returns the work counters to zero for the next launch. (Launches
    // on one context must not overlap: they share these counters.)
    __threadfence();
    if (atomicAdd(a.work + 1, 1) == (int)gridDim.x - 1) {
      atomicExch(a.work, 0);
      atomicExch(a.work + 1, 0);
    }
  }
}

}  // namespace

namespace zl {

zl_status launch_prefill_tc(zl_ctx* ctx, const void* q, const void* k, const void* v,
                            const int32_t* cu_seqlens, int num_seqs, int max_seq_len,
                            int64_t total_tokens, void* out, int H, int Hkv, int d, float scale,
                            int causal, zl_gqa_map map, cudaStream_t st) {
  if (d != D || Hkv <= 0 || H % Hkv != 0 || (H / Hkv) % NQ != 0 || total_tokens <= 0 ||
      (map != ZL_GQA_GROUPED && H != Hkv) || (H / Hkv) < NQ)
    return ZL_ERR_UNSUPPORTED;
  if (total_tokens >= (1ll << 31) || num_seqs > 0x7fffffff / (H / NQ)) return ZL_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out)) & 15)
    return ZL_ERR_UNSUPPORTED;
  const int max_tiles = (max_seq_len + BM - 1) / BM;
  if (max_tiles <= 0 || (int64_t)max_tiles * num_seqs * (H / NQ) >= (1ll << 31)) return ZL_ERR_UNSUPPORTED;
  CUtensorMap tq, tk, tv;
  zl_status s = make_tmap_bf16(&tq, q, (uint64_t)H * D, total_tokens, (uint64_t)H * D * 2, 64, BM);
  if (s != ZL_OK) return s;
  if ((s = make_tmap_bf16(&tk, k, (uint64_t)Hkv * D, total_tokens, (uint64_t)Hkv * D * 2, 64, BN)) != ZL_OK) return s;
  if ((s = make_tmap_bf16(&tv, v, (uint64_t)Hkv * D, total_tokens, (uint64_t)Hkv * D * 2, 64, BN)) != ZL_OK) return s;
  PrefillArgs args;
  args.cu_seqlens = cu_seqlens;
  args.out = (__nv_bfloat16*)out;
  args.status = ctx->d_status;
  args.work = ctx->prefill_work;
  args.total_tokens = total_tokens;
  args.H = H; args.Hkv = Hkv; args.G = H / Hkv; args.num_seqs = num_seqs;
  args.scale_log2 = scale * LOG2E;
  args.causal = causal ? 1 : 0;
  args.hp_count = H / NQ;
  args.max_tiles = max_tiles;
  args.total_items = (int)((int64_t)max_tiles * num_seqs * args.hp_count);
  // the shared-memory limit is a per-device attribute of the function
  static std::atomic<uint64_t> attr_set{0};
  if (ctx->device < 64 && !(attr_set.load() & (1ull << ctx->device))) {
    ZL_CUDA_TRY(cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Smem::kTotal));
    attr_set.fetch_or(1ull << ctx->device);
  }
  const int grid = args.total_items < ctx->num_sms ? args.total_items : ctx->num_sms;
  prefill_tc_kernel<<<grid, THREADS, Smem::kTotal, st>>>(args, tq, tk, tv);
  ZL_LAUNCH_CHECK(ctx);
  return ZL_OK;
}

}  // namespace zl
