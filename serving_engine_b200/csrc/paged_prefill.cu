// Chunked-prefill causal attention over the paged KV pool on 5th-generation
// tensor cores (tcgen05 + TMEM + TMA) for sm_100a.
//
// Replaces the prefill / mixed use (q_len > 1) of the reference's Triton kernel
// paged_flash_fwd_kernel (serving_engine/paged_attention_kernel.py:16-122), which
// runs 16x16 tiles per (q tile, row, q head) and reads the KV of a kv head once
// per q head of its GQA group.
//
// One CTA computes a 128-row tile of one prefill row and one kv head; the 128
// MMA rows pack (query, head) pairs of the GQA group, row m = query (m / G),
// head (m % G), so each K/V tile is read once for the whole group:
//   warp 0     TMA producer: the Q tile once, then K and V tiles of 128 keys
//              (8 paged blocks, gathered through the block table) into 2-stage
//              rings of 128B-swizzled K-major panels; K runs two tiles ahead of
//              V, matching the order the MMAs consume them;
//   warp 1     owns TMEM (512 columns: three S buffers at 0/128/256, O at 384)
//              and issues the MMAs from one thread: S(j+2) = Q K(j+2)^T is
//              issued before O += P(j) V(j), so two score tiles are always in
//              flight while the softmax works on a third;
//   warps 2-9  two softmax warpgroups; a thread owns half of one tile row
//              (TMEM lane): read its 64 scores, mask boundary tiles, agree on
//              the row max with its partner thread through shared memory,
//              online softmax with a lazily rescaled reference max (O and l are
//              only rescaled when a block max exceeds it by 2^8), write P as
//              bf16 to a swizzled shared-memory tile, and finally normalise its
//              half of O, store it and the LSE.
// P V is split into a 16-bit high part and its 16-bit remainder for tiles
// whose rows see fewer than kSplitBelow keys (early positions of a prompt),
// where one rounding of P would cost more than the output tolerance.
//
// Roofline: tensor. Algorithmic FLOPs per call = sum over rows, heads and
// queries of 4 * head_dim * (visible keys of that query).
#include "seb_common.cuh"
#include "seb_tcgen05.cuh"
#include "seb_tma.cuh"

#include <type_traits>

namespace seb {
namespace {

constexpr float kLn2p = 0.69314718055994530942f;
constexpr float kLog2ep = 1.44269504088896340736f;
constexpr unsigned kFullMask = 0xffffffffu;
constexpr int kBM = 128;        // MMA rows per CTA
constexpr int kBN = 128;        // keys per KV tile
constexpr int kThreads = 320;   // producer, MMA, 8 softmax warps (2 warpgroups)
constexpr int kRing = 2;        // K and V ring depths
constexpr int kSBufs = 3;       // score buffers in TMEM
constexpr int kTmemCols = 512;
constexpr int kColS = 0;        // S buffers at columns 0, 128, 256
constexpr int kColO = 384;      // O accumulator
constexpr float kLazyThreshold = 8.0f;
constexpr int kSplitBelow = 256;

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
  int32_t mtiles;  // m-tiles per row (ceil(max_q_len / queries_per_tile))
  int32_t hq, hkv, group, qpt;  // qpt = queries per tile = 128 / group
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
  static constexpr int kPanels = D / 64;
  static constexpr int kPanel = 128 * 128;  // 128 rows x 128 bytes
  static constexpr int kTileQ = kPanels * kPanel;
  static constexpr int kTileKV = kPanels * kPanel;
  static constexpr int kTileP = 2 * kPanel;  // 128 rows x 128 keys
  static constexpr int oQ = 0;
  static constexpr int oK = oQ + kTileQ;
  static constexpr int oV = oK + kRing * kTileKV;
  static constexpr int oP = oV + kRing * kTileKV;
  static constexpr int oPlo = oP + kTileP;  // P's 16-bit remainder (split tiles)
  static constexpr int oBar = oPlo + kTileP;
  static constexpr int oX = oBar + 256;  // row max / sum exchange between the two softmax warpgroups
  static constexpr int kBytes = oX + 2 * 128 * 4;
};

// mbarrier slots
enum {
  kBarQ = 0,
  kBarKFull = 1,    // +stage
  kBarVFull = 3,    // +stage
  kBarKEmpty = 5,   // +stage: S of the tile has consumed K
  kBarVEmpty = 7,   // +stage: PV of the tile has consumed V
  kBarSFull = 9,    // +S buffer (3)
  kBarSFree = 12,   // +S buffer (3)
  kBarPFull = 15,
  kBarPFree = 16,   // one completion per PV (P buffer free, O stable)
  kBarDone = 17,
  kNumBars = 18
};

// 2^x by the MUFU instruction (ex2.approx.ftz: 2^-22 relative error, -inf -> +0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ bool wait_or_flag(uint32_t bar, uint32_t parity, bool& failed) {
  if (failed) return false;
  if (!mbar_wait_bounded(bar, parity)) {
    failed = true;
    return false;
  }
  return true;
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

  // ---- tile coordinates (m-tiles of a row visited late-first: they are the longest)
  int bx = blockIdx.x;
  const int mt = p.mtiles - 1 - (bx % p.mtiles);
  bx /= p.mtiles;
  const int kvh = bx % p.hkv;
  const int prow = bx / p.hkv;
  if (prow >= p.num_prefill_rows) return;
  const int row = p.rows ? __ldg(p.rows + prow) : prow;
  if (row < 0 || row >= p.num_rows) {
    if (threadIdx.x == 0 && kvh == 0 && mt == 0) atomic_or_err(p.err, SEB_ERRBIT_META);
    return;
  }
  const int q_len = __ldg(p.q_lens + row);
  const int q_start = __ldg(p.q_starts + row);
  const int k_len = max(__ldg(p.k_lens + row), 0);
  const int qpos0 = __ldg(p.q_pos + row);
  const int i0 = mt * p.qpt;
  if (i0 >= q_len) return;
  const int i_last = min(i0 + p.qpt, q_len) - 1;
  const int ceil16 = (k_len + 15) & ~15;
  int nvis_tile = p.causal ? min(ceil16, qpos0 + i_last + 1) : ceil16;
  nvis_tile = max(nvis_tile, 0);
  int nblk = (nvis_tile + 15) >> 4;
  if (nblk > p.max_blocks) {
    if (threadIdx.x == 0) atomic_or_err(p.err, SEB_ERRBIT_KLEN);
    nblk = (int)p.max_blocks;
    nvis_tile = nblk * 16;
  }
  const int ntiles = (nblk + 7) >> 3;
  const int min_vis = p.causal ? min(ceil16, qpos0 + i0 + 1) : ceil16;
  const bool split = min_vis < kSplitBelow;
  const int G = p.group;

  // Softmax-thread row identity (also used by the no-key epilogue).
  const int q4 = warp & 3;
  const int m = q4 * 32 + lane;
  const int qi = i0 + m / G;
  const int gh = m % G;
  const bool row_valid = (warp >= 2) && qi <= i_last;

  if (ntiles == 0) {
    // No visible keys: the reference's loop never runs, O = 0/0, LSE = -inf.
    if (row_valid && warp < 6) {
      T* op = reinterpret_cast<T*>(p.out) + (int64_t)(q_start + qi) * p.o_st + (int64_t)(kvh * G + gh) * p.o_sh;
      for (int d = 0; d < D; ++d) op[d] = Elem<T>::from_float(__int_as_float(0x7fc00000));
      p.lse[(int64_t)(q_start + qi) * p.lse_st + kvh * G + gh] = -INFINITY;
    }
    return;
  }

  const uint32_t bar = base + L::oBar;  // mbarrier i at bar + 8 * i
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sbase + L::oBar + 8 * kNumBars);
  if (threadIdx.x == 0) {
    mbar_init(bar + 8 * kBarQ, 1);
    for (int s = 0; s < kRing; ++s) {
      mbar_init(bar + 8 * (kBarKFull + s), 1);
      mbar_init(bar + 8 * (kBarVFull + s), 1);
      mbar_init(bar + 8 * (kBarKEmpty + s), 1);
      mbar_init(bar + 8 * (kBarVEmpty + s), 1);
    }
    for (int b = 0; b < kSBufs; ++b) {
      mbar_init(bar + 8 * (kBarSFull + b), 1);
      mbar_init(bar + 8 * (kBarSFree + b), 8);
    }
    mbar_init(bar + 8 * kBarPFull, 8);
    mbar_init(bar + 8 * kBarPFree, 1);
    mbar_init(bar + 8 * kBarDone, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensor_map(&tmap_q);
      prefetch_tensor_map(&tmap_k);
      prefetch_tensor_map(&tmap_v);
      mbar_arrive_expect_tx(bar + 8 * kBarQ, L::kTileQ);
#pragma unroll
      for (int pn = 0; pn < L::kPanels; ++pn)
        tma_load_3d(base + L::oQ + pn * L::kPanel, &tmap_q, pn * 64, kvh * G, q_start + i0, bar + 8 * kBarQ);
    }
    const int32_t* bt = p.block_table + (int64_t)row * p.bt_stride;
    // Load K (is_v = 0) or V (is_v = 1) of tile j into stage j % 2.
    auto load = [&](int j, int is_v) -> bool {
      const int s = j & 1;
      const int u = j >> 1;
      if (u >= 1 && !wait_or_flag(bar + 8 * ((is_v ? kBarVEmpty : kBarKEmpty) + s), (u - 1) & 1, failed))
        return false;
      const int nb = min(8, nblk - 8 * j);
      int bid = 0;
      if (lane < nb) {
        bid = __ldg(bt + 8 * j + lane);
        if (bid < 0 || (int64_t)bid >= p.num_blocks) {
          atomic_or_err(p.err, SEB_ERRBIT_BLOCK_ID);
          bid = 0;  // read a real block instead; the row's result is flagged as invalid
        }
      }
      const uint32_t fb = bar + 8 * ((is_v ? kBarVFull : kBarKFull) + s);
      if (lane == 0) mbar_arrive_expect_tx(fb, nb * L::kPanels * 2048);
      __syncwarp();
      if (lane < nb) {
        const uint32_t dst = base + (is_v ? L::oV : L::oK) + s * L::kTileKV + lane * 2048;
#pragma unroll
        for (int pn = 0; pn < L::kPanels; ++pn)
          tma_load_3d(dst + pn * L::kPanel, is_v ? &tmap_v : &tmap_k, pn * 64, kvh, bid * 16, fb);
      }
      return true;
    };
    // Consumption order of the MMA warp: K(0), K(1), then per tile j K(j+2), V(j).
    int k_issued = 0, v_issued = 0;
    for (int j = 0; j < min(2, ntiles); ++j)
      if (load(j, 0)) ++k_issued;
    for (int j = 0; j < ntiles && !failed; ++j) {
      if (load(j, 1)) ++v_issued;
      if (j + 2 < ntiles && load(j + 2, 0)) ++k_issued;
    }
    // Leave no copy in flight: the last loads must have landed.
    for (int j = max(0, k_issued - kRing); j < k_issued; ++j)
      mbar_wait_bounded(bar + 8 * (kBarKFull + (j & 1)), (j >> 1) & 1, 1u << 16);
    for (int j = max(0, v_issued - kRing); j < v_issued; ++j)
      mbar_wait_bounded(bar + 8 * (kBarVFull + (j & 1)), (j >> 1) & 1, 1u << 16);
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    constexpr uint32_t idesc_qk = tc::idesc_f16(kBf16, false, kBM, kBN);
    constexpr uint32_t idesc_pv = tc::idesc_f16(kBf16, true, kBM, D);
    wait_or_flag(bar + 8 * kBarQ, 0, failed);
    auto issue_s = [&](int j) {
      const int s = j & 1;
      const int b = j % kSBufs;
      const int u = j / kSBufs;
      if (!wait_or_flag(bar + 8 * (kBarKFull + s), (j >> 1) & 1, failed)) return;
      if (u >= 1 && !wait_or_flag(bar + 8 * (kBarSFree + b), (u - 1) & 1, failed)) return;
      tc::fence_after_sync();
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t a = tc::smem_desc_sw128(base + L::oQ + (kk >> 2) * L::kPanel + (kk & 3) * 32, 16, 1024);
          const uint64_t bd =
              tc::smem_desc_sw128(base + L::oK + s * L::kTileKV + (kk >> 2) * L::kPanel + (kk & 3) * 32, 16, 1024);
          tc::mma_ss(tmem + kColS + b * kBN, a, bd, idesc_qk, kk > 0);
        }
        tc::commit(bar + 8 * (kBarSFull + b));
        tc::commit(bar + 8 * (kBarKEmpty + s));
      }
      __syncwarp();
    };
    for (int j = 0; j < min(2, ntiles) && !failed; ++j) issue_s(j);
    for (int j = 0; j < ntiles && !failed; ++j) {
      if (j + 2 < ntiles) issue_s(j + 2);
      if (failed) break;
      const int s = j & 1;
      if (!wait_or_flag(bar + 8 * (kBarVFull + s), (j >> 1) & 1, failed)) break;
      // Rows of this tile that hold real keys: loaded (nblk) and below k_len.
      const int r0 = min(max(k_len - j * kBN, 0), min(8, nblk - 8 * j) * 16);
      if (r0 < kBN) {
        // V rows of padding keys must be exact zeros (their P is 0 or, for the
        // reference's zero-padded keys, exp(-m)); the pool past k_len and the
        // rows of blocks this tile did not load may hold anything.
        char* vt = sbase + L::oV + s * L::kTileKV;
        for (int c = lane; c < (kBN - r0) * L::kPanels * 8; c += 32) {
          const int r = r0 + c / (L::kPanels * 8);
          const int rem = c % (L::kPanels * 8);
          *reinterpret_cast<uint4*>(vt + (rem >> 3) * L::kPanel + r * 128 + (rem & 7) * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
      if (!wait_or_flag(bar + 8 * kBarPFull, j & 1, failed)) break;
      tc::fence_after_sync();
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t a = tc::smem_desc_sw128(base + L::oP + (kk >> 2) * L::kPanel + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = tc::smem_desc_sw128(base + L::oV + s * L::kTileKV + kk * 2048, L::kPanel, 1024);
          tc::mma_ss(tmem + kColO, a, bd, idesc_pv, j > 0 || kk > 0);
        }
        if (split) {
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint64_t a = tc::smem_desc_sw128(base + L::oPlo + (kk >> 2) * L::kPanel + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = tc::smem_desc_sw128(base + L::oV + s * L::kTileKV + kk * 2048, L::kPanel, 1024);
            tc::mma_ss(tmem + kColO, a, bd, idesc_pv, true);
          }
        }
        tc::commit(bar + 8 * kBarPFree);
        tc::commit(bar + 8 * (kBarVEmpty + s));
      }
      __syncwarp();
    }
    // Every MMA this thread issued has completed before TMEM is released.
    if (lane == 0) tc::commit(bar + 8 * kBarDone);
    __syncwarp();
    mbar_wait_bounded(bar + 8 * kBarDone, 0, 1u << 20);
  } else {
    // ------------------------------------------------------------ softmax
    // Two warpgroups share each tile row: `half` 0 owns keys / O columns 0..D/2-1
    // of its row, half 1 the rest. Warps w and w+4 see the same TMEM lanes (w % 4).
    const int half = (warp - 2) >> 2;
    const uint32_t taddr = tmem + ((uint32_t)(q4 * 32) << 16);
    const int pos = qpos0 + qi;
    const int vis = row_valid ? (p.causal ? min(ceil16, pos + 1) : ceil16) : 0;
    const float c = p.scale_log2;
    float* xchg = reinterpret_cast<float*>(sbase + L::oX);  // [half][128]: row maxima per tile, then sums
    float m_ref = -INFINITY;
    float l = 0.f;
    char* ph = sbase + L::oP + half * L::kPanel + m * 128;
    char* pl = sbase + L::oPlo + half * L::kPanel + m * 128;
    // After a failed (timed-out) wait the loop keeps its shape with the waits
    // skipped, so both warpgroups still meet at every named barrier.
    for (int j = 0; j < ntiles; ++j) {
      const int b = j % kSBufs;
      wait_or_flag(bar + 8 * (kBarSFull + b), (j / kSBufs) & 1, failed);
      tc::fence_after_sync();
      float x[64];
      {
        float v[32];
        tc::tmem_ld32(taddr + kColS + b * kBN + half * 64, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = v[i];
        tc::tmem_ld32(taddr + kColS + b * kBN + half * 64 + 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) x[32 + i] = v[i];
      }
      tc::tmem_wait_ld();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar + 8 * (kBarSFree + b));

      // Tiles every valid row sees in full need no mask: scores stay raw and
      // the scale folds into the exponent's FMA. Boundary tiles are masked and
      // scaled here (keys past the row's visible range: -inf; zero-padded keys
      // of the last block: 0).
      const bool full = (j + 1) * kBN <= min_vis && (j + 1) * kBN <= k_len;
      float cm = c;
      if (!full) {
        const int kbase = j * kBN + half * 64;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const int key = kbase + i;
          float v = x[i] * c;
          if (key >= vis) v = -INFINITY;
          else if (key >= k_len) v = 0.f;
          x[i] = v;
        }
        cm = 1.f;
      }
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = fmaxf(x[i], x[8 + i]);
#pragma unroll
      for (int i = 16; i < 64; i += 8)
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = fmaxf(mx[k], x[i + k]);
      float mloc = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      mloc *= cm;
      // Row max over both halves (second barrier: both reads done before the
      // next tile's writes).
      xchg[half * 128 + m] = mloc;
      named_bar_sync(1 + q4, 64);
      const float mb = fmaxf(mloc, xchg[(1 - half) * 128 + m]);
      named_bar_sync(1 + q4, 64);
      const bool need = mb > m_ref + kLazyThreshold;
      float factor = 1.f;
      if (need) {
        factor = fast_exp2(m_ref - mb);  // 0 while m_ref is -inf
        l *= factor;
        m_ref = mb;
      }
      // PV(j-1) must be complete: it reads the P buffers and accumulates O.
      if (j > 0) wait_or_flag(bar + 8 * kBarPFree, (j - 1) & 1, failed);
      tc::fence_after_sync();
      if (j > 0 && __any_sync(kFullMask, need)) {
        // warp-collective: rows that keep their reference max scale by 1
#pragma unroll
        for (int cc = 0; cc < D / 64; ++cc) {
          float o[32];
          const uint32_t a = taddr + kColO + half * (D / 2) + 32 * cc;
          tc::tmem_ld32(a, o);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= factor;
          tc::tmem_st32(a, o);
        }
        tc::tmem_wait_st();
      }
      const float neg_m = m_ref == -INFINITY ? 0.f : -m_ref;
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a0 = fast_exp2(fmaf(x[8 * ch + 2 * e], cm, neg_m));
          const float a1 = fast_exp2(fmaf(x[8 * ch + 2 * e + 1], cm, neg_m));
          ls[e] += a0 + a1;
          hi[e] = Mma<T>::pack(a0, a1);
          if (split) {
            const float2 f = Mma<T>::unpack(hi[e]);
            lo[e] = Mma<T>::pack(a0 - f.x, a1 - f.y);
          }
        }
        const int off = ((ch ^ (m & 7))) << 4;
        *reinterpret_cast<uint4*>(ph + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        if (split) *reinterpret_cast<uint4*>(pl + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      fence_proxy_async_smem();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar + 8 * kBarPFull);
    }
    // ------------------------------------------------------------ epilogue
    wait_or_flag(bar + 8 * kBarPFree, (ntiles - 1) & 1, failed);
    tc::fence_after_sync();
    xchg[half * 128 + m] = l;
    named_bar_sync(1 + q4, 64);
    if (!__any_sync(kFullMask, failed)) {  // warp-uniform: tcgen05.ld is warp-collective
      const float l_tot = l + xchg[(1 - half) * 128 + m];
      const float inv = 1.f / l_tot;
      T* op = reinterpret_cast<T*>(p.out) + (int64_t)(q_start + qi) * p.o_st + (int64_t)(kvh * G + gh) * p.o_sh +
              half * (D / 2);
#pragma unroll
      for (int cc = 0; cc < D / 64; ++cc) {
        float o[32];
        tc::tmem_ld32(taddr + kColO + half * (D / 2) + 32 * cc, o);
        tc::tmem_wait_ld();
        if (row_valid) {
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) w[e] = Mma<T>::pack(o[8 * v8 + 2 * e] * inv, o[8 * v8 + 2 * e + 1] * inv);
            *reinterpret_cast<uint4*>(op + 32 * cc + 8 * v8) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      if (row_valid && half == 0)
        p.lse[(int64_t)(q_start + qi) * p.lse_st + kvh * G + gh] = m_ref * kLn2p + logf(l_tot);
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

template <typename T, int D>
int launch_prefill(const PrefillParams& p, const void* q, int64_t q_st, int64_t q_sh, int total_query,
                   const void* kc, const void* vc, cudaStream_t s) {
  using L = PrefillLayout<D>;
  constexpr int smem = L::kBytes + 1024;
  auto kern = prefill_tc_kernel<T, D>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    SEB_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set[dev] = true;
  }
  const int dtype = std::is_same<T, __nv_bfloat16>::value ? SEB_BF16 : SEB_F16;
  CUtensorMap tq, tk, tv;
  const uint64_t qdims[3] = {(uint64_t)D, (uint64_t)p.hq, (uint64_t)total_query};
  const uint64_t qstr[2] = {(uint64_t)q_sh * 2, (uint64_t)q_st * 2};
  const uint32_t qbox[3] = {64, (uint32_t)p.group, (uint32_t)p.qpt};
  int rc = tensor_map_3d(&tq, q, dtype, qdims, qstr, qbox);
  if (rc != SEB_OK) return rc;
  rc = kv_tensor_map(&tk, kc, dtype, p.num_blocks, p.hkv, D);
  if (rc != SEB_OK) return rc;
  rc = kv_tensor_map(&tv, vc, dtype, p.num_blocks, p.hkv, D);
  if (rc != SEB_OK) return rc;
  const int64_t grid = (int64_t)p.num_prefill_rows * p.hkv * p.mtiles;
  kern<<<(unsigned)grid, kThreads, smem, s>>>(p, tq, tk, tv);
  return launch_status("prefill_tc_kernel");
}

}  // namespace
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
  using namespace seb;
  clear_error();
  SEB_CHECK_ARG(dtype == SEB_BF16 || dtype == SEB_F16, "seb_paged_prefill: bf16 or fp16 required (dtype %d)", dtype);
  SEB_CHECK_ARG(num_prefill_rows >= 0 && num_rows >= 0 && total_query >= 0 && max_q_len >= 0,
                "seb_paged_prefill: negative count");
  if (num_prefill_rows == 0 || max_q_len == 0) return SEB_OK;
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
  p.mtiles = (max_q_len + p.qpt - 1) / p.qpt;
  p.scale_log2 = scale * kLog2ep;
  p.causal = is_causal ? 1 : 0;
  p.out = static_cast<char*>(out);
  p.o_st = out_stride_token;
  p.o_sh = out_stride_head;
  p.lse = lse;
  p.lse_st = lse_stride_token;
  p.err = err;
  const int64_t grid = (int64_t)num_prefill_rows * num_kv_heads * p.mtiles;
  SEB_CHECK_ARG(grid < (1ll << 31), "seb_paged_prefill: grid too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == SEB_BF16) {
    return head_dim == 128 ? launch_prefill<__nv_bfloat16, 128>(p, q, q_stride_token, q_stride_head, total_query,
                                                                k_cache, v_cache, s)
                           : launch_prefill<__nv_bfloat16, 64>(p, q, q_stride_token, q_stride_head, total_query,
                                                               k_cache, v_cache, s);
  }
  return head_dim == 128
             ? launch_prefill<__half, 128>(p, q, q_stride_token, q_stride_head, total_query, k_cache, v_cache, s)
             : launch_prefill<__half, 64>(p, q, q_stride_token, q_stride_head, total_query, k_cache, v_cache, s);
}
