// Chunked-prefill causal attention over the paged KV pool on 5th-generation
// tensor cores (tcgen05 + TMEM + TMA) for sm_100a.
//
// Replaces the prefill / mixed use (q_len > 1) of the reference's Triton kernel
// paged_flash_fwd_kernel (serving_engine/paged_attention_kernel.py:16-122), which
// runs 16x16 tiles per (q tile, row, q head) and reads the KV of a kv head once
// per q head of its GQA group.
//
// Two kernels share the work-unit definition: a unit is one prefill row, one kv
// head and a pair of 128-row Q tiles (256 MMA rows). The 128 MMA rows of a Q
// tile pack (query, head) pairs of the GQA group, row m = query (m / G), head
// (m % G), so each K/V tile is read once for the whole group. K/V tiles hold
// 128 keys (8 paged blocks), gathered through the block table by TMA as 16-row
// boxes of 128-byte panels.
//
// prefill_pair_kernel (head_dim 128) runs a unit on a cluster of two CTAs whose
// MMAs span both SMs (tcgen05 cta_group::2); it is described above the kernel.
//
// prefill_tc_kernel (head_dim 64) runs a unit in one CTA, persistent (one CTA
// per SM walks units c, c + grid, ...; Q double-buffered, the rings and barrier
// phases running on from unit to unit):
//   warp 0     TMA producer: the unit's Q tiles, then K and V tiles (block ids
//              prefetched a window ahead) into 3-stage rings;
//   warp 1     owns TMEM (512 columns: per Q tile, S of 128 columns with P
//              written over its first 64 as 16-bit pairs, O of 64 columns and
//              64 columns for P's remainder) and issues the MMAs from one
//              thread in ping-pong order: per KV tile j and Q tile
//              t, O(t) += P(t, j) V(j) (P read from TMEM), then S(t, j + 1),
//              so one Q tile's softmax runs while the other's MMAs execute;
//   warps 2-9  one softmax warpgroup per Q tile; a thread owns one tile row
//              (TMEM lane): read its 128 scores in one TMEM round trip, mask
//              boundary tiles, online softmax with a lazily rescaled reference
//              max (O and l are only rescaled when a block max exceeds it by
//              2^8), write P, and finally normalise its row of O, store it and
//              the LSE.
// P V is split into a 16-bit high part and its 16-bit remainder for units whose
// first query sees fewer than kSplitBelow keys (early positions of a prompt),
// where one rounding of P would cost more than the output tolerance.
//
// Roofline: tensor. Algorithmic FLOPs per call = sum over rows, heads and
// queries of 4 * head_dim * (visible keys of that query).
#include "seb_common.cuh"
#include "seb_tcgen05.cuh"
#include "seb_tma.cuh"

#include <algorithm>
#include <type_traits>

namespace seb {
namespace {

constexpr float kLn2p = 0.69314718055994530942f;
constexpr float kLog2ep = 1.44269504088896340736f;
constexpr unsigned kFullMask = 0xffffffffu;
constexpr int kBM = 128;       // MMA rows per Q tile
constexpr int kBN = 128;       // keys per KV tile (8 paged blocks)
constexpr int kQT = 2;         // Q tiles per CTA: each K/V tile feeds 256 rows
constexpr int kThreads = 320;  // producer, MMA, one softmax warpgroup per Q tile
constexpr int kKStages = 3;    // K ring depth (the rings run on from unit to unit)
constexpr int kVStages = 3;    // V ring depth
constexpr int kTmemCols = 512;
// TMEM columns of Q tile t (head_dim 64): S at t * 128 (128 fp32 scores per row;
// P overwrites its first 64 columns as packed 16-bit pairs), O at 256 + t * 64,
// P's 16-bit remainder (pairs whose first query sees few keys) at 384 + t * 64.
constexpr int kColS = 0;
constexpr int kColO = 256;
constexpr int kColRem = 384;
constexpr float kLazyThreshold = 8.0f;
// One 16-bit rounding of P costs up to about 0.013 / sqrt(visible keys) of
// output error (8e-4 at 260 keys, 4e-4 at 1000), which next to the output's own
// rounding (up to 9.8e-4 below |O| = 0.5 in bf16) would break a 2e-3 bound below
// about a thousand keys; units whose first query sees fewer keys than this run
// the remainder pass.
constexpr int kSplitBelow = 1024;

struct PrefillParams {
  int64_t num_blocks;
  const int32_t* block_table;
  int64_t bt_stride;
  int64_t max_blocks;
  const int32_t* q_starts;
  const int32_t* q_lens;
  const int32_t* k_lens;
  const int32_t* q_pos;
  int32_t num_rows;
  const int32_t* rows;
  int32_t num_prefill_rows;
  int32_t mpairs;  // Q-tile pairs per row: ceil(max_q_len / (2 * queries_per_tile))
  // Unit-list mode (units built on the device, seb_paged_attention): unit u is
  // row unit_list[2u], kv head unit_list[2u+1] & 255, Q-tile pair
  // unit_list[2u+1] >> 8, for u < *num_units (<= unit_cap). NULL: units come
  // from rows x kv heads x mpairs as above.
  const int32_t* unit_list;
  const int32_t* num_units;
  int32_t unit_cap;
  int32_t hq, hkv, group, qpt;  // qpt = queries per Q tile = 128 / group
  float scale_log2;
  int32_t causal;
  char* out;
  int64_t o_st, o_sh;
  float* lse;
  int64_t lse_st;
  int32_t* err;
};

template <int D>
struct PrefillLayout {
  static constexpr int kPanels = D / 64;      // 128-byte column panels of a row
  static constexpr int kPanel = 128 * 128;    // 128 rows x 128 bytes
  static constexpr int kTileQ = kPanels * kPanel;
  static constexpr int kTileKV = kPanels * kPanel;
  static constexpr int oQ = 0;                      // [Q buffer (2)][Q tile]
  static constexpr int oK = oQ + 2 * kQT * kTileQ;  // [stage]
  static constexpr int oV = oK + kKStages * kTileKV;
  static constexpr int oBar = oV + kVStages * kTileKV;
  static constexpr int kBytes = oBar + 256;
};

// mbarrier slots of prefill_tc_kernel
enum {
  kBarQFull = 0,                       // +Q buffer (2): the unit's Q tiles landed
  kBarQEmpty = 2,                      // +Q buffer: the unit's last S done, Q may be reloaded
  kBarKFull = 4,                       // +stage
  kBarKEmpty = kBarKFull + kKStages,   // +stage: S of every Q tile consumed K
  kBarVFull = kBarKEmpty + kKStages,   // +stage
  kBarVEmpty = kBarVFull + kVStages,   // +stage: PV of every Q tile consumed V
  kBarSFull = kBarVEmpty + kVStages,   // +Q tile: S(t, j) complete (and every earlier MMA)
  kBarPFull = kBarSFull + kQT,         // +Q tile: the tile's 4 softmax warps stored P(t, j)
  kBarODone = kBarPFull + kQT,         // +Q tile: the unit's last PV(t) complete, O(t) final
  kBarFinal = kBarODone + kQT,         // every MMA complete before TMEM is released
  kNumBars = kBarFinal + 1
};
static_assert(kNumBars * 8 + 8 <= 256, "barrier region");

// Barrier `id` (1..15) over `n` threads (a multiple of 32) of the CTA.
__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// 2^x by the MUFU instruction (ex2.approx.ftz: 2^-22 relative error, -inf -> +0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100 f32x2 instructions: one issue slot for the two
// lanes of an FMA, add, subtract or multiply), so that the softmax, which is
// bound by issue slots and the MUFU, spends half the slots on its fp32 work.
__device__ __forceinline__ uint64_t f2_pack(float2 v) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(v.x), "f"(v.y));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_pack(a)), "l"(f2_pack(b)), "l"(f2_pack(c)));
  return f2_unpack(d);
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_pack(a)), "l"(f2_pack(b)));
  return f2_unpack(d);
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_pack(a)), "l"(f2_pack(b)));
  return f2_unpack(d);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_pack(a)), "l"(f2_pack(b)));
  return f2_unpack(d);
}
__device__ __forceinline__ float2 splat2(float v) { return make_float2(v, v); }

// max(a, b, c) in one instruction (sm_100); NaN operands are dropped as fmaxf drops them.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for two scores on the FMA pipe, so that part of a tile's exponentials
// run beside the MUFU's. Cody-Waite range reduction: 2^x = 2^j * 2^f with
// j = rint(x) (the 1.5 * 2^23 addition leaves j in the low mantissa bits) and
// f = x - j in [-1/2, 1/2], exact; 2^f by the degree-3 polynomial that minimises
// the relative error on that interval (coefficients fitted for this kernel by a
// linear program: 7.5e-5 relative error in fp32, against 2^-9 for the 16-bit P
// it feeds). Valid for x <= 127. It is used only on unmasked tiles (no -inf
// scores); there a score more than 126 below the row's reference maximum weighs
// about 1.2e-38 instead of ex2's 0. max.NaN keeps a NaN score NaN, as ex2 does.
__device__ __forceinline__ float2 poly_exp2x2(float2 x) {
  asm("max.NaN.f32 %0, %0, 0fC2FC0000;" : "+f"(x.x));  // max(x, -126)
  asm("max.NaN.f32 %0, %0, 0fC2FC0000;" : "+f"(x.y));
  const float2 t = add2(x, splat2(12582912.f));
  const float2 f = sub2(x, sub2(t, splat2(12582912.f)));
  float2 p = fma2(splat2(0x1.c3f76p-5f), f, splat2(0x1.f0de1ap-3f));
  p = fma2(p, f, splat2(0x1.62f31ap-1f));
  p = fma2(p, f, splat2(0x1.fff692p-1f));
  const float2 scale = make_float2(__int_as_float((__float_as_int(t.x) << 23) + 0x3f800000),
                                   __int_as_float((__float_as_int(t.y) << 23) + 0x3f800000));  // 2^j
  return mul2(p, scale);
}

// Pairs of a 32-score chunk (bit e: scores 2e, 2e + 1) whose exponentials the
// pair kernel evaluates with poly_exp2 on unmasked tiles of pairs without the
// remainder pass: 5 of 16. Config 3 on one box, 100 steps, two runs each:
// 3 of 16 (0x4210) 932.6 / 933.4 TFLOP/s, 4 (0x8888) 972.2 / 971.4, 5 (0x8A22)
// 979.2 / 978.8, 6 (0x9249) 912.9 / 912.7.
#ifndef SEB_POLY_PAIRS
#define SEB_POLY_PAIRS 0x8A22u
#endif
constexpr unsigned kPolyPairs = SEB_POLY_PAIRS;

__device__ __forceinline__ bool wait_or_flag(uint32_t bar, uint32_t parity, bool& failed) {
  if (failed) return false;
  if (!mbar_wait_bounded(bar, parity)) {
    failed = true;
    return false;
  }
  return true;
}

// The same for the CTA-pair kernel, whose barriers are completed from the
// other SM of the pair: short suspensions, bounded at about one second.
__device__ __forceinline__ bool wait_or_flag_cluster(uint32_t bar, uint32_t parity, bool& failed) {
  if (failed) return false;
  if (mbar_test_wait(bar, parity)) return true;
  for (uint32_t i = 0; i < (1u << 23); ++i)
    if (mbar_try_wait_hint(bar, parity, 128)) return true;
  failed = true;
  return false;
}

// Scores of keys [key0, key0 + 32) of one row, masked in place when the tile is
// not fully visible: keys past the row's visible range -> -inf, the reference's
// zero-padded keys of the last block (past k_len) -> 0; scaled by c when masked.
__device__ __forceinline__ void mask_chunk(float (&x)[32], int key0, int vis, int k_len, float c) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int key = key0 + i;
    float v = x[i] * c;
    if (key >= vis) v = -INFINITY;
    else if (key >= k_len) v = 0.f;
    x[i] = v;
  }
}

// Causal masking of raw (unscaled) scores of a row whose visible keys all lie
// below k_len: keys at or past the row's visible end -> -inf. The positive
// scale is applied afterwards (-inf stays -inf), one compare and select a score.
__device__ __forceinline__ void mask_chunk_causal(float (&x)[32], int key0, int vis) {
  const int lim = vis - key0;
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] = i < lim ? x[i] : -INFINITY;
}

// One work unit (prefill row, kv head, pair of Q tiles), decoded identically by
// every role of either kernel.
struct PairUnit {
  int row, kvh, q_len, q_start, k_len, qpos0, ceil16, pair0, i_last, nblk, ntiles;
  bool split;
};

// Decodes unit u; false: the unit does nothing (no such row or pair). Without a
// unit list, a row's pairs are visited late-first (they are the longest).
__device__ __forceinline__ bool pair_unit(const PrefillParams& p, int u, PairUnit& w) {
  int pr;
  if (p.unit_list) {
    w.row = __ldg(p.unit_list + 2 * u);
    const int e = __ldg(p.unit_list + 2 * u + 1);
    w.kvh = e & 255;
    pr = e >> 8;
  } else {
    pr = p.mpairs - 1 - (u % p.mpairs);
    u /= p.mpairs;
    w.kvh = u % p.hkv;
    const int prow = u / p.hkv;
    if (prow >= p.num_prefill_rows) return false;
    w.row = p.rows ? __ldg(p.rows + prow) : prow;
  }
  if (w.row < 0 || w.row >= p.num_rows) return false;
  w.q_len = __ldg(p.q_lens + w.row);
  w.q_start = __ldg(p.q_starts + w.row);
  w.k_len = max(__ldg(p.k_lens + w.row), 0);
  w.qpos0 = __ldg(p.q_pos + w.row);
  w.ceil16 = (w.k_len + 15) & ~15;
  w.pair0 = pr * kQT * p.qpt;
  if (w.pair0 >= w.q_len) return false;
  w.i_last = min(w.pair0 + kQT * p.qpt, w.q_len) - 1;
  w.split = (p.causal ? min(w.ceil16, w.qpos0 + w.pair0 + 1) : w.ceil16) < kSplitBelow;
  const int nvis = max(p.causal ? min(w.ceil16, w.qpos0 + w.i_last + 1) : w.ceil16, 0);
  w.nblk = min((nvis + 15) >> 4, (int)p.max_blocks);
  w.ntiles = (w.nblk + 7) >> 3;
  return true;
}

// Metadata errors of units first, first + stride, ... (a row index outside the
// batch; a row whose keys need more blocks than the block table holds), each
// reported by the CTA that owns the row's first unit of a kv head or its last
// pair. The builder of a unit list checks its rows itself.
__device__ __forceinline__ void report_unit_errors(const PrefillParams& p, int first, int stride, int units) {
  if (p.unit_list) return;
  for (int u = first; u < units; u += stride) {
    const int prow = (u / p.mpairs) / p.hkv;
    const int row = p.rows ? __ldg(p.rows + prow) : prow;
    if (u % (p.mpairs * p.hkv) == 0 && (row < 0 || row >= p.num_rows)) atomic_or_err(p.err, SEB_ERRBIT_META);
    if (row >= 0 && row < p.num_rows && (u % p.mpairs) == p.mpairs - 1) {
      const int k_len = max(__ldg(p.k_lens + row), 0);
      if (((k_len + 15) >> 4) > p.max_blocks && (u / p.mpairs) % p.hkv == 0) atomic_or_err(p.err, SEB_ERRBIT_KLEN);
    }
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v) {
  using L = PrefillLayout<D>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ __align__(1024) char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  char* sbase = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  static_assert(D == 64, "TMEM layout for head_dim 64 (O and P's remainder: 64 columns per Q tile)");
  // Persistent: CTA c walks the work units c, c + gridDim.x, ... with its Q
  // buffers, K/V rings and barrier phases running on from unit to unit, so the
  // next unit's Q and first K/V tiles load while the current unit finishes.
  // Every thread reads the same unit count, so all roles walk the same units.
  const int units = p.unit_list ? min(__ldg(p.num_units), p.unit_cap) : p.num_prefill_rows * p.hkv * p.mpairs;
  const int G = p.group;

  const uint32_t bar = base + L::oBar;  // mbarrier i at bar + 8 * i
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sbase + L::oBar + 8 * kNumBars);
  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar + 8 * (kBarQFull + b), 1);
      mbar_init(bar + 8 * (kBarQEmpty + b), 1);
    }
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(bar + 8 * (kBarKFull + s), 1);
      mbar_init(bar + 8 * (kBarKEmpty + s), 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(bar + 8 * (kBarVFull + s), 1);
      mbar_init(bar + 8 * (kBarVEmpty + s), 1);
    }
    for (int t = 0; t < kQT; ++t) {
      mbar_init(bar + 8 * (kBarSFull + t), 1);
      mbar_init(bar + 8 * (kBarPFull + t), 4);
      mbar_init(bar + 8 * (kBarODone + t), 1);
    }
    mbar_init(bar + 8 * kBarFinal, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  bool failed = false;
  PairUnit w;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensor_map(&tmap_q);
      prefetch_tensor_map(&tmap_k);
      prefetch_tensor_map(&tmap_v);
    }
    int gk = 0, gv = 0;  // K and V tiles loaded so far (ring positions)
    int nq = 0;          // units whose Q was loaded so far (Q buffer nq & 1)
    for (int u = blockIdx.x; u < units && !failed; u += gridDim.x) {
      if (!pair_unit(p, u, w) || w.ntiles == 0) continue;
      const int nqt = w.pair0 + p.qpt < w.q_len ? 2 : 1;  // Q tiles of the unit
      // Q into buffer nq & 1 once the S MMAs of the unit two back have read it.
      const int qb = nq & 1;
      if (nq >= 2 && !wait_or_flag(bar + 8 * (kBarQEmpty + qb), ((nq >> 1) - 1) & 1, failed)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(bar + 8 * (kBarQFull + qb), nqt * L::kTileQ);
        for (int t = 0; t < nqt; ++t)
#pragma unroll
          for (int pn = 0; pn < L::kPanels; ++pn)
            tma_load_3d(base + L::oQ + (qb * kQT + t) * L::kTileQ + pn * L::kPanel, &tmap_q, pn * 64, w.kvh * G,
                        w.q_start + w.pair0 + t * p.qpt, bar + 8 * (kBarQFull + qb));
      }
      __syncwarp();
      ++nq;
      const int32_t* bt = p.block_table + (int64_t)w.row * p.bt_stride;
      const int nblk = w.nblk;
      // Block ids are read a window of 4 tiles (32 blocks, one per lane) ahead of
      // their use, so the copies never wait on a block-table load. K and V keep
      // their own windows.
      auto fetch = [&](int win) -> int {
        const int blk = 32 * win + lane;
        return blk < nblk ? __ldg(bt + blk) : 0;
      };
      int kcur = fetch(0), knext = fetch(1), kw = 0;
      int vcur = kcur, vnext = knext, vw = 0;
      auto block_id = [&](int t, int& cur, int& next, int& win) -> int {
        while (win < (t >> 2)) {
          cur = next;
          next = fetch(win + 2);
          ++win;
        }
        return __shfl_sync(kFullMask, cur, ((t & 3) << 3) + (lane & 7));
      };
      // Load K (is_v = 0) or V (is_v = 1) of tile j (8 blocks) into its ring stage.
      auto load = [&](int j, int is_v) -> bool {
        const int stages = is_v ? kVStages : kKStages;
        const int g = is_v ? gv : gk;
        const int s = g % stages;
        const int uu = g / stages;
        int bid = is_v ? block_id(j, vcur, vnext, vw) : block_id(j, kcur, knext, kw);
        if (uu >= 1 && !wait_or_flag(bar + 8 * ((is_v ? kBarVEmpty : kBarKEmpty) + s), (uu - 1) & 1, failed))
          return false;
        const int nb = min(8, nblk - 8 * j);
        if (lane < nb && (bid < 0 || (int64_t)bid >= p.num_blocks)) {
          atomic_or_err(p.err, SEB_ERRBIT_BLOCK_ID);
          bid = 0;  // read a real block instead; the row's result is flagged as invalid
        }
        const uint32_t fb = bar + 8 * ((is_v ? kBarVFull : kBarKFull) + s);
        if (lane == 0) mbar_arrive_expect_tx(fb, nb * L::kPanels * 2048);
        __syncwarp();
        if (lane < nb) {
          const uint32_t dst = base + (is_v ? L::oV : L::oK) + s * L::kTileKV + lane * 2048;
#pragma unroll
          for (int pn = 0; pn < L::kPanels; ++pn)
            tma_load_3d(dst + pn * L::kPanel, is_v ? &tmap_v : &tmap_k, pn * 64, w.kvh, bid * 16, fb);
        }
        if (is_v) ++gv;
        else ++gk;
        return true;
      };
      // The MMA warp consumes K(0), then per tile j V(j) and K(j+1).
      for (int j = 0; j < w.ntiles; ++j)
        if (!load(j, 0) || !load(j, 1)) break;
    }
    // Leave no copy in flight: the last loads must have landed.
    for (int i = max(0, nq - 2); i < nq; ++i)
      mbar_wait_bounded(bar + 8 * (kBarQFull + (i & 1)), (i >> 1) & 1, 1u << 16);
    for (int i = max(0, gk - kKStages); i < gk; ++i)
      mbar_wait_bounded(bar + 8 * (kBarKFull + i % kKStages), (i / kKStages) & 1, 1u << 16);
    for (int i = max(0, gv - kVStages); i < gv; ++i)
      mbar_wait_bounded(bar + 8 * (kBarVFull + i % kVStages), (i / kVStages) & 1, 1u << 16);
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    constexpr uint32_t idesc_qk = tc::idesc_f16(kBf16, false, kBM, kBN);
    constexpr uint32_t idesc_pv = tc::idesc_f16(kBf16, true, kBM, D);
    // Metadata errors of this CTA's units, one unit per lane, while the first
    // Q and K tiles load.
    report_unit_errors(p, blockIdx.x + lane * gridDim.x, 32 * gridDim.x, units);
    // S(t) = Q(t) K^T from Q buffer qb and K stage s into the S/P columns of Q tile t.
    auto issue_s = [&](int t, int qb, int s) {
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t a = tc::smem_desc_sw128(
              base + L::oQ + (qb * kQT + t) * L::kTileQ + (kk >> 2) * L::kPanel + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = tc::smem_desc_sw128(
              base + L::oK + s * L::kTileKV + (kk >> 2) * L::kPanel + (kk & 3) * 32, 16, 1024);
          tc::mma_ss(tmem + kColS + t * 128, a, bd, idesc_qk, kk > 0);
        }
        tc::commit(bar + 8 * (kBarSFull + t));
      }
      __syncwarp();
    };
    // O(t) += P(t) V from V stage s, P read from TMEM (first: O(t) = P(t) V).
    auto issue_pv = [&](int t, int s, bool first, bool split) {
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t bd = tc::smem_desc_sw128(base + L::oV + s * L::kTileKV + kk * 2048, L::kPanel, 1024);
          tc::mma_ts(tmem + kColO + t * D, tmem + kColS + t * 128 + 8 * kk, bd, idesc_pv, !first || kk > 0);
        }
        if (split) {  // P's remainder, from its own columns
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint64_t bd = tc::smem_desc_sw128(base + L::oV + s * L::kTileKV + kk * 2048, L::kPanel, 1024);
            tc::mma_ts(tmem + kColO + t * D, tmem + kColRem + t * 64 + 8 * kk, bd, idesc_pv, true);
          }
        }
      }
      __syncwarp();
    };
    int gk = 0, gv = 0, nq = 0;
    uint32_t pphase = 0;  // bit t: parity of Q tile t's next P arrival
    // Ping-pong: per KV tile j and Q tile t, PV(t, j) then S(t, j+1), so one Q
    // tile's softmax runs while the other tile's MMAs execute. S(t, j+1)
    // overwrites the columns PV(t, j) reads P from; both are issued by this one
    // thread, and the tensor pipe runs one thread's MMAs in issue order, so
    // S(t, j+1) follows PV(t, j) at once (no wait for PV(t, j) to complete).
    // The same holds across units: the next unit's S(t, 0) follows this unit's
    // last PV(t, j), and its PV(t, 0), which overwrites O(t), waits for the
    // tile's P arrival, which the softmax posts after it read O(t).
    for (int u = blockIdx.x; u < units && !failed; u += gridDim.x) {
      if (!pair_unit(p, u, w) || w.ntiles == 0) continue;
      const int nqt = w.pair0 + p.qpt < w.q_len ? 2 : 1;
      const int qb = nq & 1;
      if (!wait_or_flag(bar + 8 * (kBarQFull + qb), (nq >> 1) & 1, failed)) break;
      ++nq;
      {
        const int sk = gk % kKStages;
        if (!wait_or_flag(bar + 8 * (kBarKFull + sk), (gk / kKStages) & 1, failed)) break;
        tc::fence_after_sync();
        for (int t = 0; t < nqt; ++t) issue_s(t, qb, sk);
        if (lane == 0) {
          tc::commit(bar + 8 * (kBarKEmpty + sk));
          if (w.ntiles == 1) tc::commit(bar + 8 * (kBarQEmpty + qb));
        }
        __syncwarp();
        ++gk;
      }
      for (int j = 0; j < w.ntiles && !failed; ++j) {
        const int sv = gv % kVStages;
        if (!wait_or_flag(bar + 8 * (kBarVFull + sv), (gv / kVStages) & 1, failed)) break;
        // Rows of this tile that hold real keys: loaded (nblk) and below k_len.
        const int r0 = min(max(w.k_len - j * kBN, 0), min(8, w.nblk - 8 * j) * 16);
        if (r0 < kBN) {
          // V rows of padding keys must be exact zeros (their P is 0 or, for the
          // reference's zero-padded keys, exp(-m)); the pool past k_len and the
          // rows of blocks this tile did not load may hold anything.
          char* vt = sbase + L::oV + sv * L::kTileKV;
          for (int c = lane; c < (kBN - r0) * L::kPanels * 8; c += 32) {
            const int r = r0 + c / (L::kPanels * 8);
            const int rem = c % (L::kPanels * 8);
            *reinterpret_cast<uint4*>(vt + (rem >> 3) * L::kPanel + r * 128 + (rem & 7) * 16) = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
          __syncwarp();
        }
        const bool next = j + 1 < w.ntiles;
        const int sk = gk % kKStages;
        for (int t = 0; t < nqt && !failed; ++t) {
          if (!wait_or_flag(bar + 8 * (kBarPFull + t), (pphase >> t) & 1u, failed)) break;
          pphase ^= 1u << t;
          tc::fence_after_sync();
          issue_pv(t, sv, j == 0, w.split);
          if (!next) {
            if (lane == 0) tc::commit(bar + 8 * (kBarODone + t));
            __syncwarp();
            continue;
          }
          if (t == 0 && !wait_or_flag(bar + 8 * (kBarKFull + sk), (gk / kKStages) & 1, failed)) break;
          tc::fence_after_sync();
          issue_s(t, qb, sk);
        }
        if (lane == 0) {
          tc::commit(bar + 8 * (kBarVEmpty + sv));
          if (next) {
            tc::commit(bar + 8 * (kBarKEmpty + sk));
            if (j + 2 == w.ntiles) tc::commit(bar + 8 * (kBarQEmpty + qb));
          }
        }
        __syncwarp();
        ++gv;
        if (next) ++gk;
      }
    }
    // Every MMA this thread issued has completed before TMEM is released.
    if (lane == 0) tc::commit(bar + 8 * kBarFinal);
    __syncwarp();
    mbar_wait_bounded(bar + 8 * kBarFinal, 0, 1u << 20);
  } else {
    // ------------------------------------------------------------ softmax
    // Warpgroup qt owns Q tile qt of every unit that has it; a thread owns one
    // MMA row (TMEM lane) m = query (m / G), head (m % G).
    const int qt = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int m = q4 * 32 + lane;
    const uint32_t taddr = tmem + ((uint32_t)(q4 * 32) << 16);
    const uint32_t col_s = kColS + qt * 128;
    const uint32_t col_o = kColO + qt * D;
    const float c = p.scale_log2;
    int ns = 0;  // S tiles of Q tile qt consumed so far (parity of kBarSFull + qt)
    int nu = 0;  // units of Q tile qt finished so far (parity of kBarODone + qt)
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      if (!pair_unit(p, u, w)) continue;
      const int nqt = w.pair0 + p.qpt < w.q_len ? 2 : 1;
      if (qt >= nqt) continue;
      const int i0 = w.pair0 + qt * p.qpt;  // first query of this Q tile
      const int qi = i0 + m / G;
      const int gh = m % G;
      const bool row_valid = qi <= w.i_last;
      T* op = reinterpret_cast<T*>(p.out) + (int64_t)(w.q_start + qi) * p.o_st + (int64_t)(w.kvh * G + gh) * p.o_sh;
      float* lp = p.lse + (int64_t)(w.q_start + qi) * p.lse_st + w.kvh * G + gh;
      if (w.ntiles == 0) {
        // No visible keys: the reference's loop never runs, O = 0/0, LSE = -inf.
        if (row_valid) {
          for (int d = 0; d < D; ++d) op[d] = Elem<T>::from_float(__int_as_float(0x7fc00000));
          *lp = -INFINITY;
        }
        continue;
      }
      const int pos = w.qpos0 + qi;
      const int vis = row_valid ? (p.causal ? min(w.ceil16, pos + 1) : w.ceil16) : 0;
      const int min_vis = p.causal ? min(w.ceil16, w.qpos0 + i0 + 1) : w.ceil16;
      float m_ref = -INFINITY;
      float l = 0.f;
      // After a failed (timed-out) wait the loop keeps its shape with the waits
      // skipped; warp-collective TMEM accesses stay warp-uniform.
      for (int j = 0; j < w.ntiles; ++j, ++ns) {
        // S(t, j) complete; its commit also covers PV(t, j-1), so O is stable.
        wait_or_flag(bar + 8 * (kBarSFull + qt), ns & 1, failed);
        tc::fence_after_sync();
        // Tiles every valid row of the Q tile sees in full need no mask: scores
        // stay raw and the (positive) scale folds into the row max and the
        // exponent's FMA. Any other scale takes the masked path, which scales first.
        const bool full = c > 0.f && (j + 1) * kBN <= min_vis && (j + 1) * kBN <= w.k_len;
        const float cm = full ? c : 1.f;
        // The row's 128 scores in one TMEM round trip.
        float x[4][32];
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) tc::tmem_ld32(taddr + col_s + 32 * ch, x[ch]);
        tc::tmem_wait_ld();
        if (!full) {
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) mask_chunk(x[ch], j * kBN + 32 * ch, vis, w.k_len, c);
        }
        float mx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = fmaxf(fmaxf(x[0][i], x[0][8 + i]), fmaxf(x[0][16 + i], x[0][24 + i]));
#pragma unroll
        for (int ch = 1; ch < 4; ++ch)
#pragma unroll
          for (int i = 0; i < 8; ++i)
            mx[i] = fmaxf(mx[i], fmaxf(fmaxf(x[ch][i], x[ch][8 + i]), fmaxf(x[ch][16 + i], x[ch][24 + i])));
        const float mb =
            cm * fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        const bool need = mb > m_ref + kLazyThreshold;
        float factor = 1.f;
        if (need) {
          factor = fast_exp2(m_ref - mb);  // 0 while m_ref is -inf
          l *= factor;
          m_ref = mb;
        }
        // P = 2^(s - m) as 16-bit pairs over the first 64 S columns (already read),
        // its remainder (split pairs) in the tile's remainder columns.
        const float neg_m = m_ref == -INFINITY ? 0.f : -m_ref;
        float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          {
            uint32_t hi[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float a0 = fast_exp2(fmaf(x[ch][2 * e], cm, neg_m));
              const float a1 = fast_exp2(fmaf(x[ch][2 * e + 1], cm, neg_m));
              ls[e & 3] += a0 + a1;
              hi[e] = Mma<T>::pack(a0, a1);
              x[ch][2 * e] = a0;  // probabilities replace the consumed scores
              x[ch][2 * e + 1] = a1;
            }
            tc::tmem_st16u(taddr + col_s + 16 * ch, hi);
          }
          if (w.split) {  // remainder p - round16(p), recomputed from the probabilities
            uint32_t lo[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float2 f = Mma<T>::unpack(Mma<T>::pack(x[ch][2 * e], x[ch][2 * e + 1]));
              lo[e] = Mma<T>::pack(x[ch][2 * e] - f.x, x[ch][2 * e + 1] - f.y);
            }
            tc::tmem_st16u(taddr + kColRem + qt * 64 + 16 * ch, lo);
          }
        }
        l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
        // O is stable (the S commit covers PV(t, j-1)); PV(t, j) is issued only
        // after this thread's P arrival, so the rescale may come last.
        if (j > 0 && __any_sync(kFullMask, need)) {
          // warp-collective: rows that keep their reference max scale by 1
#pragma unroll 1
          for (int cc = 0; cc < D / 16; ++cc) {
            float o[16];
            const uint32_t a = taddr + col_o + 16 * cc;
            tc::tmem_ld16(a, o);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] *= factor;
            tc::tmem_st16(a, o);
          }
        }
        tc::tmem_wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar + 8 * (kBarPFull + qt));
      }
      // ---------------------------------------------------------- epilogue
      // The unit's last PV of this Q tile has completed: O is final.
      wait_or_flag(bar + 8 * (kBarODone + qt), nu & 1, failed);
      ++nu;
      tc::fence_after_sync();
      if (__any_sync(kFullMask, failed)) break;  // warp-uniform: tcgen05.ld is warp-collective
      const float inv = 1.f / l;
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        float o[32];
        tc::tmem_ld32(taddr + col_o + 32 * cc, o);
        tc::tmem_wait_ld();
        if (row_valid) {
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            uint32_t wv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) wv[e] = Mma<T>::pack(o[8 * v8 + 2 * e] * inv, o[8 * v8 + 2 * e + 1] * inv);
            *reinterpret_cast<uint4*>(op + 32 * cc + 8 * v8) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
          }
        }
      }
      if (row_valid) *lp = m_ref * kLn2p + logf(l);
      // The next unit's first PV overwrites O: order this warp's O loads before
      // its next P arrival.
      tc::fence_before_sync();
    }
  }

  if (failed && lane == 0) atomic_or_err(p.err, SEB_ERRBIT_TIMEOUT);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair kernel (head_dim 128). A cluster of two CTAs on two SMs computes
// the 256 MMA rows of a pair of Q tiles with every MMA spanning both SMs
// (tcgen05 cta_group::2, M = 256): CTA r holds Q rows [128 r, 128 r + 128) and
// their S and O in its own TMEM; of each 128-key tile it loads half of K (keys
// [64 r, 64 r + 64)) and half of V (head dims [64 r, 64 r + 64)). Per SM that
// halves the operand bytes the tensor core reads from shared memory for 128 MMA
// rows, and it frees TMEM for three S buffers per SM: S(j + 3) is issued as soon
// as P V(j) has released its buffer, so the softmax finds its next scores ready
// and runs back to back.
// The kernel is persistent: one cluster per SM pair walks the work units
// (prefill row, kv head, pair of Q tiles) c, c + C, c + 2C, ... with its K/V
// rings, S buffers and their barrier phases running on from unit to unit, and Q
// double-buffered, so the next unit's Q and first K/V tiles load while the
// current unit finishes.
//   warp 0     TMA producer of its CTA's Q tile and K halves; warp 10 of its V
//              halves. Both complete their bytes on the even CTA's barriers;
//   warp 11    (even CTA) issues S(j) once K(j) landed and P V(j - 3) released
//              S buffer j % 3; warp 1 (even CTA) issues P V(j) once V(j) landed
//              and both CTAs wrote P(j). Their commits arrive on both CTAs';
//   warps 2-9  softmax of the CTA's 128 rows in two warpgroups, one per half
//              (64 keys) of a tile, so two warps share each sub-partition: a
//              thread owns one row of its half, the halves exchange row maxima
//              through shared memory, P goes over the buffer's first 64 columns
//              and, for pairs whose first query sees fewer than kSplitBelow
//              keys, P's 16-bit remainder over the next 64 (read already).
constexpr int kPairThreads = 384;
constexpr int kPairVWarp = 10;   // V producer
constexpr int kPairSWarp = 11;   // S = Q K^T issuer
constexpr int kPairKStages = 3;
constexpr int kPairVStages = 4;
constexpr int kPairColO = 384;   // O: columns [384, 512); S buffer b: [128 b, 128 b + 128)

struct PairLayout {
  static constexpr int kPanelQ = 128 * 128;    // 128 rows x 128 bytes
  static constexpr int kTileQ = 2 * kPanelQ;   // 128 rows x 128 dims
  static constexpr int kPanelK = 64 * 128;     // 64 keys x 128 bytes
  static constexpr int kStageK = 2 * kPanelK;  // 64 keys x 128 dims
  static constexpr int kStageV = 128 * 128;    // 128 keys x 64 dims
  static constexpr int oQ = 0;                 // [2 buffers]
  static constexpr int oK = oQ + 2 * kTileQ;
  static constexpr int oV = oK + kPairKStages * kStageK;
  static constexpr int oO = oV + kPairVStages * kStageV;  // O staged for its TMA store: one panel per half
  static constexpr int oBar = oO + kTileQ;
  static constexpr int oX = oBar + 512;        // [tile parity][half][row] row maxima; row sums at unit ends
  static constexpr int kBytes = oX + 2 * 2 * 128 * 4;
};

enum {
  kPBarQFull = 0,                              // +buffer (2), even CTA: both Q halves landed
  kPBarQEmpty = 2,                             // +buffer, both CTAs: the unit's last S done
  kPBarKFull = 4,                              // +stage (3), even CTA: both K halves landed
  kPBarKEmpty = kPBarKFull + kPairKStages,     // +stage, both CTAs: S of the tile done
  kPBarVFull = kPBarKEmpty + kPairKStages,     // +stage (4), even CTA: two arrivals (one per CTA)
  kPBarVEmpty = kPBarVFull + kPairVStages,     // +stage, both CTAs
  kPBarSFull = kPBarVEmpty + kPairVStages,     // +buffer (3), both CTAs
  kPBarPFull = kPBarSFull + 3,                 // +buffer, even CTA: 16 softmax warps wrote P
  kPBarPFree = kPBarPFull + 3,                 // +buffer, both CTAs: P V of the buffer done
  kPBarDone = kPBarPFree + 3,                  // both CTAs: a final commit of each issuing warp
  kPBarVLand = kPBarDone + 1,                  // local: this CTA's V half of a unit's last tile landed
  kPNumBars = kPBarVLand + 1
};
static_assert(kPNumBars * 8 + 16 <= 512, "barrier region");

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    prefill_pair_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tmap_q,
                        const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                        const __grid_constant__ CUtensorMap tmap_o) {
  using L = PairLayout;
  constexpr int D = 128;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ __align__(1024) char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  char* sbase = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const int cid = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;
  // Every thread of both CTAs reads the same unit count, so all roles walk the
  // same units.
  const int units = p.unit_list ? min(__ldg(p.num_units), p.unit_cap) : p.num_prefill_rows * p.hkv * p.mpairs;
  const int G = p.group;


  const uint32_t bar = base + L::oBar;        // this CTA's mbarrier i at bar + 8 i
  const uint32_t lead = mapa_shared(bar, 0);  // the even CTA's
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sbase + L::oBar + 8 * kPNumBars);
  if (threadIdx.x == 0) {
    for (int q = 0; q < 2; ++q) {
      mbar_init(bar + 8 * (kPBarQFull + q), 1);
      mbar_init(bar + 8 * (kPBarQEmpty + q), 1);
    }
    for (int s = 0; s < kPairKStages; ++s) {
      mbar_init(bar + 8 * (kPBarKFull + s), 1);
      mbar_init(bar + 8 * (kPBarKEmpty + s), 1);
    }
    for (int s = 0; s < kPairVStages; ++s) {
      mbar_init(bar + 8 * (kPBarVFull + s), 2);
      mbar_init(bar + 8 * (kPBarVEmpty + s), 1);
    }
    for (int b = 0; b < 3; ++b) {
      mbar_init(bar + 8 * (kPBarSFull + b), 1);
      mbar_init(bar + 8 * (kPBarPFull + b), 16);
      mbar_init(bar + 8 * (kPBarPFree + b), 1);
    }
    mbar_init(bar + 8 * kPBarDone, 2);
    mbar_init(bar + 8 * kPBarVLand, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
    tc::tmem_relinquish_pair();
  }
  tc::fence_before_sync();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc::fence_after_sync();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  bool failed = false;
  PairUnit w;

  if (warp == 0 || warp == kPairVWarp) {
    // ------------------------------------------------------------ producers
    if (warp == 0 && lane == 0) {
      prefetch_tensor_map(&tmap_q);
      prefetch_tensor_map(&tmap_k);
    }
    if (warp == kPairVWarp && lane == 0) prefetch_tensor_map(&tmap_v);
    int g = 0;       // tiles loaded so far (ring position)
    int nq = 0;      // Q tiles loaded so far
    int nland = 0;   // V tiles patched through the local barrier so far
    for (int u = cid; u < units && !failed; u += nclusters) {
      if (!pair_unit(p, u, w) || w.ntiles == 0) continue;
      const int32_t* bt = p.block_table + (int64_t)w.row * p.bt_stride;
      const int nblk = w.nblk;
      auto fetch = [&](int win) -> int {
        const int blk = 32 * win + lane;
        return blk < nblk ? __ldg(bt + blk) : 0;
      };
      auto checked = [&](int bid) -> int {
        if (bid < 0 || (int64_t)bid >= p.num_blocks) {
          atomic_or_err(p.err, SEB_ERRBIT_BLOCK_ID);
          return 0;  // read a real block instead; the row's result is flagged as invalid
        }
        return bid;
      };
      int cur = fetch(0), nxt = fetch(1), win = 0;
      if (warp == 0) {
        const int qb = nq & 1;
        if (nq >= 2 && !wait_or_flag_cluster(bar + 8 * (kPBarQEmpty + qb), ((nq >> 1) - 1) & 1, failed)) break;
        if (lane == 0) {
          if (crank == 0) mbar_arrive_expect_tx(bar + 8 * (kPBarQFull + qb), 2 * L::kTileQ);
#pragma unroll
          for (int pn = 0; pn < 2; ++pn)
            tma_load_3d_pair(base + L::oQ + qb * L::kTileQ + pn * L::kPanelQ, &tmap_q, pn * 64, w.kvh * G,
                             w.q_start + w.pair0 + (int)crank * p.qpt, lead + 8 * (kPBarQFull + qb));
        }
        ++nq;
      }
      for (int j = 0; j < w.ntiles && !failed; ++j, ++g) {
        while (win < (j >> 2)) {
          cur = nxt;
          nxt = fetch(win + 2);
          ++win;
        }
        const int nb_all = min(8, nblk - 8 * j);
        if (warp == 0) {
          // K(j): this CTA's 4 blocks (keys [64 crank, 64 crank + 64)), both panels
          const int s = g % kPairKStages, uu = g / kPairKStages;
          int bid = __shfl_sync(kFullMask, cur, ((j & 3) << 3) + ((4 * (int)crank + (lane & 3)) & 7));
          if (uu >= 1 && !wait_or_flag_cluster(bar + 8 * (kPBarKEmpty + s), (uu - 1) & 1, failed)) break;
          const int nb = min(4, max(0, nb_all - 4 * (int)crank));
          if (lane == 0 && crank == 0) mbar_arrive_expect_tx(bar + 8 * (kPBarKFull + s), nb_all * 2 * 2048);
          __syncwarp();
          if (lane < nb) {
            bid = checked(bid);
            const uint32_t dst = base + L::oK + s * L::kStageK + lane * 2048;
#pragma unroll
            for (int pn = 0; pn < 2; ++pn)
              tma_load_3d_pair(dst + pn * L::kPanelK, &tmap_k, pn * 64, w.kvh, bid * 16,
                               lead + 8 * (kPBarKFull + s));
          }
        } else {
          // V(j): all 8 blocks, this CTA's 64 head dims. A tile whose rows past
          // k_len (or past the loaded blocks) must read as zeros lands on a local
          // barrier first, is patched, and then reported.
          const int s = g % kPairVStages, uu = g / kPairVStages;
          int bid = __shfl_sync(kFullMask, cur, ((j & 3) << 3) + (lane & 7));
          if (uu >= 1 && !wait_or_flag_cluster(bar + 8 * (kPBarVEmpty + s), (uu - 1) & 1, failed)) break;
          const int r0 = min(max(w.k_len - j * kBN, 0), nb_all * 16);
          const uint32_t dst = base + L::oV + s * L::kStageV;
          const uint32_t full_bar = bar + 8 * (kPBarVFull + s);
          if (r0 == kBN) {
            if (lane == 0 && crank == 0) mbar_arrive_expect_tx(full_bar, 2 * 8 * 2048);
            __syncwarp();
            if (lane < 8)
              tma_load_3d_pair(dst + lane * 2048, &tmap_v, (int)crank * 64, w.kvh, checked(bid) * 16,
                               lead + 8 * (kPBarVFull + s));
            if (lane == 0 && crank == 1) mbar_arrive_cluster(lead + 8 * (kPBarVFull + s));
          } else {
            if (lane == 0) mbar_arrive_expect_tx(bar + 8 * kPBarVLand, nb_all * 2048);
            __syncwarp();
            if (lane < nb_all)
              tma_load_3d(dst + lane * 2048, &tmap_v, (int)crank * 64, w.kvh, checked(bid) * 16,
                          bar + 8 * kPBarVLand);
            if (!wait_or_flag_cluster(bar + 8 * kPBarVLand, nland & 1, failed)) break;
            ++nland;
            char* vt = sbase + L::oV + s * L::kStageV;
            for (int c = lane; c < (kBN - r0) * 8; c += 32)
              *reinterpret_cast<uint4*>(vt + (r0 + c / 8) * 128 + (c % 8) * 16) = make_uint4(0, 0, 0, 0);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (crank == 0) mbar_arrive(full_bar);
              else mbar_arrive_cluster(lead + 8 * (kPBarVFull + s));
            }
          }
        }
      }
    }
    // No copy may still be in flight when the pair exits: the even CTA's full
    // barriers count the bytes of both CTAs.
    if (crank == 0) {
      bool drain_failed = false;
      const int stages = warp == 0 ? kPairKStages : kPairVStages;
      const int fb = warp == 0 ? kPBarKFull : kPBarVFull;
      for (int i = max(0, g - stages); i < g; ++i)
        wait_or_flag_cluster(bar + 8 * (fb + i % stages), (i / stages) & 1, drain_failed);
    }
  } else if (warp == 1 || warp == kPairSWarp) {
    // ---------------------------------------------------------------- MMA
    if (crank == 0) {
      constexpr uint32_t idesc_qk = tc::idesc_f16(kBf16, false, 256, kBN);
      constexpr uint32_t idesc_pv = tc::idesc_f16(kBf16, true, 256, D);
      int g = 0, nq = 0;
      for (int u = cid; u < units && !failed; u += nclusters) {
        if (!pair_unit(p, u, w) || w.ntiles == 0) continue;
        if (warp == kPairSWarp) {
          // S(j) = Q K(j)^T into S buffer g % 3
          const int qb = nq & 1;
          if (!wait_or_flag_cluster(bar + 8 * (kPBarQFull + qb), (nq >> 1) & 1, failed)) break;
          for (int j = 0; j < w.ntiles && !failed; ++j, ++g) {
            const int b = g % 3, s = g % kPairKStages;
            if (!wait_or_flag_cluster(bar + 8 * (kPBarKFull + s), (g / kPairKStages) & 1, failed)) break;
            if (g >= 3 && !wait_or_flag_cluster(bar + 8 * (kPBarPFree + b), ((g - 3) / 3) & 1, failed)) break;
            // A unit's first S waits for the previous unit's last P V, so that P V
            // (whose completion the previous unit's epilogue waits on) is not
            // queued behind it on the tensor pipe.
            if (j == 0 && g >= 1 &&
                !wait_or_flag_cluster(bar + 8 * (kPBarPFree + (g - 1) % 3), ((g - 1) / 3) & 1, failed))
              break;
            tc::fence_after_sync();
            if (lane == 0) {
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk) {
                const uint64_t a = tc::smem_desc_sw128(
                    base + L::oQ + qb * L::kTileQ + (kk >> 2) * L::kPanelQ + (kk & 3) * 32, 16, 1024);
                const uint64_t bd = tc::smem_desc_sw128(
                    base + L::oK + s * L::kStageK + (kk >> 2) * L::kPanelK + (kk & 3) * 32, 16, 1024);
                tc::mma_ss_pair(tmem + 128 * b, a, bd, idesc_qk, kk > 0);
              }
              tc::commit_pair(bar + 8 * (kPBarSFull + b), 3);
              tc::commit_pair(bar + 8 * (kPBarKEmpty + s), 3);
              if (j == w.ntiles - 1) tc::commit_pair(bar + 8 * (kPBarQEmpty + qb), 3);
            }
            __syncwarp();
          }
          ++nq;
        } else {
          // O += P(j) V(j), P read from TMEM (and its remainder for split pairs)
          for (int j = 0; j < w.ntiles && !failed; ++j, ++g) {
            const int b = g % 3, s = g % kPairVStages;
            if (!wait_or_flag_cluster(bar + 8 * (kPBarVFull + s), (g / kPairVStages) & 1, failed)) break;
            if (!wait_or_flag_cluster(bar + 8 * (kPBarPFull + b), (g / 3) & 1, failed)) break;
            tc::fence_after_sync();
            if (lane == 0) {
#pragma unroll
              for (int kk = 0; kk < kBN / 16; ++kk) {
                const uint64_t bd =
                    tc::smem_desc_sw128(base + L::oV + s * L::kStageV + kk * 2048, L::kStageV, 1024);
                tc::mma_ts_pair(tmem + kPairColO, tmem + 128 * b + 8 * kk, bd, idesc_pv, j > 0 || kk > 0);
              }
              if (w.split) {
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk) {
                  const uint64_t bd =
                      tc::smem_desc_sw128(base + L::oV + s * L::kStageV + kk * 2048, L::kStageV, 1024);
                  tc::mma_ts_pair(tmem + kPairColO, tmem + 128 * b + 64 + 8 * kk, bd, idesc_pv, true);
                }
              }
              tc::commit_pair(bar + 8 * (kPBarPFree + b), 3);
              tc::commit_pair(bar + 8 * (kPBarVEmpty + s), 3);
            }
            __syncwarp();
          }
        }
      }
      // Every MMA this warp issued has completed before either CTA releases TMEM.
      if (lane == 0) tc::commit_pair(bar + 8 * kPBarDone, 3);
      __syncwarp();
    } else if (warp == 1) {
      // The odd CTA's warp 1 issues nothing: it reports the metadata errors of
      // the pair's units, one unit per lane, once per unit.
      report_unit_errors(p, cid + lane * nclusters, 32 * nclusters, units);
    }
    bool done_failed = false;
    wait_or_flag_cluster(bar + 8 * kPBarDone, 0, done_failed);
  } else if (warp < kPairVWarp) {
    // ------------------------------------------------------------ softmax
    const int q4 = warp & 3;
    const int khalf = (warp - 2) >> 2;  // which 64 keys of a tile
    const int m = q4 * 32 + lane;
    const int kh0 = 64 * khalf;
    const uint32_t taddr = tmem + ((uint32_t)(q4 * 32) << 16);
    const float c = p.scale_log2;
    float* xchg = reinterpret_cast<float*>(sbase + L::oX);  // [parity][half][row]
    int g = 0;
    for (int u = cid; u < units; u += nclusters) {
      if (!pair_unit(p, u, w)) continue;
      const int i0 = w.pair0 + (int)crank * p.qpt;  // this CTA's first query
      const int qi = i0 + m / G;
      const int gh = m % G;
      const bool row_valid = qi <= w.i_last;
      T* op = reinterpret_cast<T*>(p.out) + (int64_t)(w.q_start + qi) * p.o_st + (int64_t)(w.kvh * G + gh) * p.o_sh;
      float* lp = p.lse + (int64_t)(w.q_start + qi) * p.lse_st + w.kvh * G + gh;
      if (w.ntiles == 0) {
        // No visible keys: the reference's loop never runs, O = 0/0, LSE = -inf.
        if (row_valid) {
          for (int d = kh0; d < kh0 + 64; ++d) op[d] = Elem<T>::from_float(__int_as_float(0x7fc00000));
          if (khalf == 0) *lp = -INFINITY;
        }
        continue;
      }
      const int vis = row_valid ? (p.causal ? min(w.ceil16, w.qpos0 + qi + 1) : w.ceil16) : 0;
      const int min_vis = p.causal ? min(w.ceil16, w.qpos0 + i0 + 1) : w.ceil16;
      // Scores stay raw (the scale folds into the row max and the exponent's
      // FMA) on unmasked tiles and, for causal rows that see no key past k_len,
      // on masked ones too; that needs a positive scale.
      const bool pos_scale = c > 0.f;
      const bool causal_raw = pos_scale && p.causal && w.qpos0 + w.q_len <= w.k_len;
      float m_ref = -INFINITY;
      float l = 0.f;
      for (int j = 0; j < w.ntiles; ++j, ++g) {
        const int b = g % 3;
        const uint32_t col_s = 128 * b;
        wait_or_flag_cluster(bar + 8 * (kPBarSFull + b), (g / 3) & 1, failed);
        tc::fence_after_sync();
        const bool full = pos_scale && (j + 1) * kBN <= min_vis && (j + 1) * kBN <= w.k_len;
        const bool raw = full || causal_raw;
        const float cm = raw ? c : 1.f;
        float x[2][32];
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) tc::tmem_ld32(taddr + col_s + kh0 + 32 * ch, x[ch]);
        tc::tmem_wait_ld();
        if (!full) {
          if (raw) {
#pragma unroll
            for (int ch = 0; ch < 2; ++ch) mask_chunk_causal(x[ch], j * kBN + kh0 + 32 * ch, vis);
          } else {
#pragma unroll
            for (int ch = 0; ch < 2; ++ch) mask_chunk(x[ch], j * kBN + kh0 + 32 * ch, vis, w.k_len, c);
          }
        }
        float mx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          mx[i] = fmax3(fmax3(x[0][i], x[0][8 + i], x[0][16 + i]), fmax3(x[0][24 + i], x[1][i], x[1][8 + i]),
                        fmaxf(x[1][16 + i], x[1][24 + i]));
        const float mh = cm * fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
        // Row max over both halves. The barrier also orders both halves' S loads
        // before either half's P stores (P of keys 64-127 lands on S columns of
        // keys 32-63, the remainder on those of keys 64-127).
        float* xm = xchg + (g & 1) * 256;
        xm[khalf * 128 + m] = mh;
        tc::fence_before_sync();
        named_bar_sync(1 + q4, 64);
        tc::fence_after_sync();
        const float mb = fmaxf(mh, xm[(1 - khalf) * 128 + m]);
        const bool need = mb > m_ref + kLazyThreshold;
        float factor = 1.f;
        if (need) {
          factor = fast_exp2(m_ref - mb);
          l *= factor;
          m_ref = mb;
        }
        const float neg_m = m_ref == -INFINITY ? 0.f : -m_ref;
        float2 ls[4] = {splat2(0.f), splat2(0.f), splat2(0.f), splat2(0.f)};
        // P of the tile's 64 scores of this row: exponentials, row sum, 16-bit
        // P into the S buffer (and its remainder for split pairs). Unmasked
        // tiles of unsplit pairs take kPolyPairs' share on the FMA pipe.
        auto exponentiate = [&](auto poly_tag) {
          constexpr bool kPoly = decltype(poly_tag)::value;
          const float2 cm2 = splat2(cm), nm2 = splat2(neg_m);
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            {
              uint32_t hi[16];
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                const float2 y = fma2(make_float2(x[ch][2 * e], x[ch][2 * e + 1]), cm2, nm2);
                float2 a;
                if (kPoly && ((kPolyPairs >> e) & 1u)) a = poly_exp2x2(y);
                else a = make_float2(fast_exp2(y.x), fast_exp2(y.y));
                ls[e & 3] = add2(ls[e & 3], a);
                hi[e] = Mma<T>::pack(a.x, a.y);
                x[ch][2 * e] = a.x;
                x[ch][2 * e + 1] = a.y;
              }
              tc::tmem_st16u(taddr + col_s + kh0 / 2 + 16 * ch, hi);
            }
            if (!kPoly && w.split) {
              uint32_t lo[16];
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                const float2 f = Mma<T>::unpack(Mma<T>::pack(x[ch][2 * e], x[ch][2 * e + 1]));
                lo[e] = Mma<T>::pack(x[ch][2 * e] - f.x, x[ch][2 * e + 1] - f.y);
              }
              tc::tmem_st16u(taddr + col_s + 64 + kh0 / 2 + 16 * ch, lo);
            }
          }
        };
        if (kPolyPairs != 0u && full && !w.split) exponentiate(std::true_type{});
        else exponentiate(std::false_type{});
        const float2 ls2 = add2(add2(ls[0], ls[1]), add2(ls[2], ls[3]));
        l += ls2.x + ls2.y;
        if (j > 0 && __any_sync(kFullMask, need)) {
          // O must hold P V(j - 1) before it is rescaled; each half scales its 64 dims
          const int gp = g - 1;
          wait_or_flag_cluster(bar + 8 * (kPBarPFree + gp % 3), (gp / 3) & 1, failed);
          tc::fence_after_sync();
#pragma unroll 1
          for (int cc = 0; cc < 4; ++cc) {
            float o[16];
            const uint32_t a = taddr + kPairColO + kh0 + 16 * cc;
            tc::tmem_ld16(a, o);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] *= factor;
            tc::tmem_st16(a, o);
          }
        }
        tc::tmem_wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          if (crank == 0) mbar_arrive(bar + 8 * (kPBarPFull + b));
          else mbar_arrive_cluster(lead + 8 * (kPBarPFull + b));
        }
      }
      // ---------------------------------------------------------- epilogue
      // Row sums of both halves: the first barrier puts every read of the last
      // tile's maxima behind us (the sums reuse the parity-0 slots).
      named_bar_sync(1 + q4, 64);
      xchg[khalf * 128 + m] = l;
      named_bar_sync(1 + q4, 64);
      l += xchg[(1 - khalf) * 128 + m];
      named_bar_sync(1 + q4, 64);  // the next unit's first maxima may overwrite the sums
      // O is final once P V of the unit's last tile has completed.
      const int gl = g - 1;
      wait_or_flag_cluster(bar + 8 * (kPBarPFree + gl % 3), (gl / 3) & 1, failed);
      tc::fence_after_sync();
      const bool ok = !__any_sync(kFullMask, failed);
      const float inv = 1.f / l;
      if (i0 + p.qpt <= w.q_len) {
        // Every row of the tile is a query of this row: O goes through shared
        // memory, each thread's 64 values as one 128-byte row of its half's
        // panel (128B-swizzled, as the output map expects), and out in one TMA
        // store per half instead of 32 scattered rows per warp instruction.
        const bool issuer = (warp & 3) == 2 && lane == 0;  // warps 2 and 6
        if (issuer) bulk_wait_read_all();                  // the previous unit's store has read the panel
        named_bar_sync(5 + khalf, 128);
        char* panel = sbase + L::oO + khalf * L::kPanelQ;
        if (ok) {
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            float o[32];
            tc::tmem_ld32(taddr + kPairColO + kh0 + 32 * cc, o);
            tc::tmem_wait_ld();
#pragma unroll
            for (int v8 = 0; v8 < 4; ++v8) {
              uint32_t wv[4];
#pragma unroll
              for (int e = 0; e < 4; ++e)
                wv[e] = Mma<T>::pack(o[8 * v8 + 2 * e] * inv, o[8 * v8 + 2 * e + 1] * inv);
              const int chunk = (4 * cc + v8) ^ (m & 7);
              *reinterpret_cast<uint4*>(panel + m * 128 + chunk * 16) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            }
          }
        }
        fence_proxy_async_smem();
        named_bar_sync(5 + khalf, 128);
        if (issuer && ok) {
          tma_store_3d(&tmap_o, smem_u32(panel), kh0, w.kvh * G, w.q_start + i0);
          bulk_commit_group();
        }
      } else if (ok) {
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          float o[32];
          tc::tmem_ld32(taddr + kPairColO + kh0 + 32 * cc, o);
          tc::tmem_wait_ld();
          if (row_valid) {
#pragma unroll
            for (int v8 = 0; v8 < 4; ++v8) {
              uint32_t wv[4];
#pragma unroll
              for (int e = 0; e < 4; ++e)
                wv[e] = Mma<T>::pack(o[8 * v8 + 2 * e] * inv, o[8 * v8 + 2 * e + 1] * inv);
              *reinterpret_cast<uint4*>(op + kh0 + 32 * cc + 8 * v8) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            }
          }
        }
      }
      if (ok && row_valid && khalf == 0) *lp = m_ref * kLn2p + logf(l);
      // The next unit's first P V overwrites O: order this warp's O loads before
      // its next P arrival.
      tc::fence_before_sync();
    }
    if ((warp & 3) == 2 && lane == 0) bulk_wait_all();  // O stores complete before the CTA exits
  }

  if (failed && lane == 0) atomic_or_err(p.err, SEB_ERRBIT_TIMEOUT);
  tc::fence_before_sync();
  cluster_sync();  // neither CTA leaves while the pair's MMAs or copies may touch it
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc_pair(tmem, kTmemCols);
  }
}

template <typename T>
int launch_prefill_pair(const PrefillParams& p, const void* q, int64_t q_st, int64_t q_sh, int total_query,
                        const void* kc, const void* vc, cudaStream_t s) {
  constexpr int smem = PairLayout::kBytes + 1024;
  constexpr auto kern = prefill_pair_kernel<T>;
  int rc = set_smem_limit_once<kern>(smem);
  if (rc != SEB_OK) return rc;
  const int dtype = std::is_same<T, __nv_bfloat16>::value ? SEB_BF16 : SEB_F16;
  CUtensorMap tq, tk, tv;
  const uint64_t qdims[3] = {128, (uint64_t)p.hq, (uint64_t)total_query};
  const uint64_t qstr[2] = {(uint64_t)q_sh * 2, (uint64_t)q_st * 2};
  const uint32_t qbox[3] = {64, (uint32_t)p.group, (uint32_t)p.qpt};
  rc = tensor_map_3d(&tq, q, dtype, qdims, qstr, qbox);
  if (rc != SEB_OK) return rc;
  rc = kv_tensor_map(&tk, kc, dtype, p.num_blocks, p.hkv, 128);
  if (rc != SEB_OK) return rc;
  rc = kv_tensor_map(&tv, vc, dtype, p.num_blocks, p.hkv, 128);
  if (rc != SEB_OK) return rc;
  // O of a whole Q tile, stored as Q was loaded: (64 dims, group heads, qpt queries) boxes
  CUtensorMap to;
  const uint64_t ostr[2] = {(uint64_t)p.o_sh * 2, (uint64_t)p.o_st * 2};
  rc = tensor_map_3d(&to, p.out, dtype, qdims, ostr, qbox);
  if (rc != SEB_OK) return rc;
  // persistent: one cluster per pair of SMs (or per unit, when there are fewer)
  const int64_t units = p.unit_list ? (int64_t)p.unit_cap : (int64_t)p.num_prefill_rows * p.hkv * p.mpairs;
  const int64_t clusters = std::min<int64_t>(units, num_sms() / 2);
  kern<<<(unsigned)(2 * clusters), kPairThreads, smem, s>>>(p, tq, tk, tv, to);
  return launch_status("prefill_pair_kernel");
}

template <typename T, int D>
int launch_prefill(const PrefillParams& p, const void* q, int64_t q_st, int64_t q_sh, int total_query,
                   const void* kc, const void* vc, cudaStream_t s) {
  using L = PrefillLayout<D>;
  constexpr int smem = L::kBytes + 1024;
  constexpr auto kern = prefill_tc_kernel<T, D>;
  int rc = set_smem_limit_once<kern>(smem);
  if (rc != SEB_OK) return rc;
  const int dtype = std::is_same<T, __nv_bfloat16>::value ? SEB_BF16 : SEB_F16;
  CUtensorMap tq, tk, tv;
  const uint64_t qdims[3] = {(uint64_t)D, (uint64_t)p.hq, (uint64_t)total_query};
  const uint64_t qstr[2] = {(uint64_t)q_sh * 2, (uint64_t)q_st * 2};
  const uint32_t qbox[3] = {64, (uint32_t)p.group, (uint32_t)p.qpt};
  rc = tensor_map_3d(&tq, q, dtype, qdims, qstr, qbox);
  if (rc != SEB_OK) return rc;
  rc = kv_tensor_map(&tk, kc, dtype, p.num_blocks, p.hkv, D);
  if (rc != SEB_OK) return rc;
  rc = kv_tensor_map(&tv, vc, dtype, p.num_blocks, p.hkv, D);
  if (rc != SEB_OK) return rc;
  // persistent: one CTA per SM (or per unit, when there are fewer)
  const int64_t units = p.unit_list ? (int64_t)p.unit_cap : (int64_t)p.num_prefill_rows * p.hkv * p.mpairs;
  const int64_t grid = std::min<int64_t>(units, num_sms());
  kern<<<(unsigned)grid, kThreads, smem, s>>>(p, tq, tk, tv);
  return launch_status("prefill_tc_kernel");
}

}  // namespace

int paged_prefill_impl(const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* k_cache,
                       const void* v_cache, int64_t num_blocks, const int32_t* block_table,
                       int64_t block_table_stride, int64_t max_blocks, const int32_t* q_starts,
                       const int32_t* q_lens, const int32_t* k_lens, const int32_t* q_pos_offsets, int32_t num_rows,
                       int32_t total_query, const int32_t* rows, int32_t num_prefill_rows, int32_t max_q_len,
                       int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t dtype, float scale,
                       int32_t is_causal, void* out, int64_t out_stride_token, int64_t out_stride_head, float* lse,
                       int64_t lse_stride_token, int32_t* err, void* stream, const int32_t* unit_list,
                       const int32_t* num_units, int32_t unit_cap) {
  SEB_CHECK_ARG(dtype == SEB_BF16 || dtype == SEB_F16, "seb_paged_prefill: bf16 or fp16 required (dtype %d)", dtype);
  SEB_CHECK_ARG(num_prefill_rows >= 0 && num_rows >= 0 && total_query >= 0 && max_q_len >= 0 && unit_cap >= 0,
                "seb_paged_prefill: negative count");
  SEB_CHECK_ARG((unit_list == nullptr) == (num_units == nullptr), "seb_paged_prefill: unit list without its count");
  if (unit_list ? unit_cap == 0 : (num_prefill_rows == 0 || max_q_len == 0)) return SEB_OK;
  SEB_CHECK_ARG(num_q_heads > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
                "seb_paged_prefill: num_q_heads (%d) must be a positive multiple of num_kv_heads (%d)", num_q_heads,
                num_kv_heads);
  const int group = num_q_heads / num_kv_heads;
  if (!(group == 1 || group == 2 || group == 4 || group == 8 || group == 16)) {
    set_error("seb_paged_prefill: GQA group %d not supported (1, 2, 4, 8, 16)", group);
    return SEB_EUNSUPPORTED;
  }
  if (head_dim != 64 && head_dim != 128) {
    set_error("seb_paged_prefill: head_dim %d not supported (64, 128)", head_dim);
    return SEB_EUNSUPPORTED;
  }
  SEB_CHECK_ARG(q && k_cache && v_cache && block_table && q_starts && q_lens && k_lens && q_pos_offsets && out && lse,
                "seb_paged_prefill: NULL pointer argument");
  SEB_CHECK_ARG(num_blocks > 0 && max_blocks > 0 && block_table_stride >= max_blocks,
                "seb_paged_prefill: bad block table shape");
  SEB_CHECK_ARG(aligned(q, 16) && q_stride_token % 8 == 0 && q_stride_head % 8 == 0 &&
                    q_stride_head >= head_dim && q_stride_token >= q_stride_head * num_q_heads,
                "seb_paged_prefill: q must be 16-byte aligned with head stride >= head_dim and token stride >= "
                "heads x head stride, both multiples of 8 elements");
  SEB_CHECK_ARG(aligned(out, 16) && out_stride_token % 8 == 0 && out_stride_head % 8 == 0,
                "seb_paged_prefill: out must be 16-byte aligned with strides that are multiples of 8 elements");
  SEB_CHECK_ARG(aligned(k_cache, 16) && aligned(v_cache, 16), "seb_paged_prefill: KV pool not 16-byte aligned");
  PrefillParams p;
  p.num_blocks = num_blocks;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.max_blocks = max_blocks;
  p.q_starts = q_starts;
  p.q_lens = q_lens;
  p.k_lens = k_lens;
  p.q_pos = q_pos_offsets;
  p.num_rows = num_rows;
  p.rows = rows;
  p.num_prefill_rows = num_prefill_rows;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.group = group;
  p.qpt = 128 / group;
  p.mpairs = (max_q_len + kQT * p.qpt - 1) / (kQT * p.qpt);
  p.scale_log2 = scale * kLog2ep;
  p.causal = is_causal ? 1 : 0;
  p.out = static_cast<char*>(out);
  p.o_st = out_stride_token;
  p.o_sh = out_stride_head;
  p.lse = lse;
  p.lse_st = lse_stride_token;
  p.err = err;
  p.unit_list = unit_list;
  p.num_units = num_units;
  p.unit_cap = unit_list ? unit_cap : 0;
  const int64_t grid = unit_list ? (int64_t)unit_cap : (int64_t)num_prefill_rows * num_kv_heads * p.mpairs;
  SEB_CHECK_ARG(grid < (1ll << 31), "seb_paged_prefill: grid too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // head_dim 128: the CTA-pair kernel; head_dim 64: one persistent CTA per SM, a pair of Q tiles per unit
  if (dtype == SEB_BF16) {
    return head_dim == 128 ? launch_prefill_pair<__nv_bfloat16>(p, q, q_stride_token, q_stride_head, total_query,
                                                                k_cache, v_cache, s)
                           : launch_prefill<__nv_bfloat16, 64>(p, q, q_stride_token, q_stride_head, total_query,
                                                               k_cache, v_cache, s);
  }
  return head_dim == 128
             ? launch_prefill_pair<__half>(p, q, q_stride_token, q_stride_head, total_query, k_cache, v_cache, s)
             : launch_prefill<__half, 64>(p, q, q_stride_token, q_stride_head, total_query, k_cache, v_cache, s);
}

}  // namespace seb

extern "C" int seb_paged_prefill(const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* k_cache,
                                 const void* v_cache, int64_t num_blocks, const int32_t* block_table,
                                 int64_t block_table_stride, int64_t max_blocks, const int32_t* q_starts,
                                 const int32_t* q_lens, const int32_t* k_lens, const int32_t* q_pos_offsets,
                                 int32_t num_rows, int32_t total_query, const int32_t* rows,
                                 int32_t num_prefill_rows, int32_t max_q_len, int32_t num_q_heads,
                                 int32_t num_kv_heads, int32_t head_dim, int32_t dtype, float scale,
                                 int32_t is_causal, void* out, int64_t out_stride_token, int64_t out_stride_head,
                                 float* lse, int64_t lse_stride_token, int32_t* err, void* stream) {
  seb::clear_error();
  return seb::paged_prefill_impl(q, q_stride_token, q_stride_head, k_cache, v_cache, num_blocks, block_table,
                                 block_table_stride, max_blocks, q_starts, q_lens, k_lens, q_pos_offsets, num_rows,
                                 total_query, rows, num_prefill_rows, max_q_len, num_q_heads, num_kv_heads,
                                 head_dim, dtype, scale, is_causal, out, out_stride_token, out_stride_head, lse,
                                 lse_stride_token, err, stream, nullptr, nullptr, 0);
}
