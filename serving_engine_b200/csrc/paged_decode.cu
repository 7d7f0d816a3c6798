// Split-K paged decode attention for sm_100a.
//
// Replaces the decode use (q_len = 1) of the reference's Triton kernel
// paged_flash_fwd_kernel (serving_engine/paged_attention_kernel.py:16-122), which
// runs one program per (16-query tile, row, q-head), re-reads the KV of a kv head
// once per q-head of its GQA group and walks a row's whole context serially.
//
// Design (one warp = one work item (query item, kv head, split)):
//   * A split is <= 64 consecutive 16-token blocks of the row; the warp keeps the
//     split's block ids in two registers per lane and streams each block's K and
//     V tiles (TMA tiled loads of 16 rows x 128-byte swizzled panels) through a
//     STAGES-deep shared-memory ring completed on mbarriers.
//   * All query heads of the GQA group share each KV tile: the 16 keys of a block
//     are the M dimension of an m16n8k16 tensor-core tile and the (<= 8) heads of
//     the group its N dimension, so S^T = K Q^T and O^T += V^T P^T each take
//     head_dim/16 MMAs per block; P^T is moved from the accumulator layout to the
//     operand layout with movmatrix. KV is read from HBM exactly once.
//   * Online softmax in the log2 domain; per-split (m, l, O) go to a workspace
//     and the last warp to finish a split of an (item, kv head) merges them (an
//     arrival counter per item and kv head, cleared by a small memset on the
//     call's stream before the launch). Items with one split write O/LSE directly.
//
// fp32 (and any shape the tensor-core path does not cover) runs a CUDA-core
// variant with the same work decomposition and workspace format.
//
// Roofline: HBM. Algorithmic bytes = sum_items k_len * num_kv_heads * head_dim *
// 2 (K and V) * elem; each KV byte is read once regardless of the group size.
#include "seb_common.cuh"
#include "seb_tma.cuh"

#include <cmath>
#include <mutex>
#include <type_traits>

namespace seb {
namespace {

constexpr float kLn2 = 0.69314718055994530942f;
constexpr float kLog2e = 1.44269504088896340736f;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kMaxBps = 64;  // blocks per split: two block ids per lane

struct DecodeParams {
  const char* q;
  int64_t q_st, q_sh;  // elements
  const char* k_cache;
  const char* v_cache;
  int64_t num_blocks;
  const int32_t* block_table;
  int64_t bt_stride;
  int64_t max_blocks;
  const int32_t* q_starts;
  const int32_t* k_lens;
  const int32_t* q_pos;
  int32_t num_rows;
  int32_t total_query;
  const int32_t* item_query;
  const int32_t* item_row;
  int32_t num_items;
  const int32_t* num_items_dev;  // when set: only items < *num_items_dev (<= num_items) run
  int32_t hq, hkv, group;
  float scale_log2;
  int32_t causal;
  int32_t bps, max_splits;
  char* out;
  int64_t o_st, o_sh;  // elements
  float* lse;
  int64_t lse_st;
  float* ws_o;   // [items][hq][max_splits][D]
  float* ws_ml;  // [items][hq][max_splits][2]  (m in log2 units, l)
  int32_t* counters;  // [items][hkv] splits finished; cleared before each launch
  int32_t* err;
};

struct ItemInfo {
  int qtok, row, k_len, n_vis, nblk, n_splits;
  bool ok;
};

// Last row r with q_starts[r] <= qtok (rows with q_len = 0 share the start of
// the next row, so "last" picks the row that owns the token).
__device__ __forceinline__ int find_row(const DecodeParams& p, int qtok) {
  int lo = 0, hi = p.num_rows - 1, ans = 0;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(p.q_starts + mid) <= qtok) {
      ans = mid;
      lo = mid + 1;
    } else {
      hi = mid - 1;
    }
  }
  return ans;
}

// Keys visible to the item's query, following paged_attention_kernel.py:79-109:
// the reference visits ceil(k_len/16) blocks, zero-pads keys past k_len inside the
// last block (boundary-checked loads) and, when causal, drops keys after the
// query's logical position (the -1e6 bias underflows exp to exactly 0).
__device__ __forceinline__ ItemInfo item_info(const DecodeParams& p, int item) {
  ItemInfo it;
  it.ok = true;
  it.qtok = p.item_query ? __ldg(p.item_query + item) : item;
  if (it.qtok < 0 || it.qtok >= p.total_query) {
    it.ok = false;
    it.row = it.k_len = it.n_vis = it.nblk = it.n_splits = 0;
    return it;
  }
  it.row = p.item_row ? __ldg(p.item_row + item) : find_row(p, it.qtok);
  if (it.row < 0 || it.row >= p.num_rows) {
    it.ok = false;
    it.k_len = it.n_vis = it.nblk = it.n_splits = 0;
    return it;
  }
  it.k_len = max(__ldg(p.k_lens + it.row), 0);
  const int q_idx = __ldg(p.q_pos + it.row) + (it.qtok - __ldg(p.q_starts + it.row));
  const int ceil16 = (it.k_len + 15) & ~15;
  int nvis = p.causal ? min(ceil16, q_idx + 1) : ceil16;
  nvis = max(nvis, 0);
  int nblk = (nvis + 15) >> 4;
  if (nblk > p.max_blocks) {
    nblk = (int)p.max_blocks;
    nvis = nblk * 16;
  }
  it.n_vis = nvis;
  it.nblk = nblk;
  it.n_splits = (nblk + p.bps - 1) / p.bps;
  return it;
}

// Work unit of global warp w: the kv head varies fastest, then the split, then
// the item. The warps of one CTA thus share an (item, split) and are live or
// idle together (a split past the row's length exits at once), so a CTA never
// holds its shared-memory ring for one working warp while its others idle; and
// they read the same block ids, whose kv-head tiles are neighbours in the pool.
__device__ __forceinline__ int64_t unit_of_warp(const DecodeParams& p, int64_t w, int& kvh, int& split) {
  kvh = (int)(w % p.hkv);
  const int64_t tmp = w / p.hkv;
  split = (int)(tmp % p.max_splits);
  return tmp / p.max_splits;
}

__device__ __forceinline__ void report_item(const DecodeParams& p, const ItemInfo& it, int lane) {
  if (lane != 0) return;
  if (!it.ok) atomic_or_err(p.err, SEB_ERRBIT_META);
  else if ((int64_t)((it.k_len + 15) >> 4) > p.max_blocks) atomic_or_err(p.err, SEB_ERRBIT_KLEN);
}

// Block ids of blocks [b0, b0 + nb) of the row (nb <= 64): lane l holds blocks
// b0 + l and b0 + 32 + l; -1 when out of range.
struct BlockIds {
  int lo, hi;
  // Id of block b0 + j (j warp-uniform).
  __device__ __forceinline__ int get(int j) const { return __shfl_sync(0xffffffffu, j < 32 ? lo : hi, j & 31); }
};

__device__ __forceinline__ int load_block_id(const DecodeParams& p, const ItemInfo& it, int blk) {
  int bid = __ldg(p.block_table + (int64_t)it.row * p.bt_stride + blk);
  if (bid < 0 || (int64_t)bid >= p.num_blocks) {
    atomic_or_err(p.err, SEB_ERRBIT_BLOCK_ID);
    bid = -1;
  }
  return bid;
}

__device__ __forceinline__ BlockIds load_block_ids(const DecodeParams& p, const ItemInfo& it, int b0, int nb,
                                                   int lane) {
  BlockIds ids{-1, -1};
  if (lane < nb) ids.lo = load_block_id(p, it, b0 + lane);
  if (lane + 32 < nb) ids.hi = load_block_id(p, it, b0 + 32 + lane);
  return ids;
}

// --------------------------------------------------------------------------
// Split-K merge, run by the last warp to finish a split of an (item, kv head).
// Up to 32 splits are merged for 4 query heads of the group at a time: lane s
// loads split s's (m, l) of all 4 heads at once and turns them into weights
// 2^(m_s - M); then each lane owns D/32 consecutive head dims and sums the
// weighted partial O of every split, with the loads of 4 heads x KU splits in
// flight together. Partials written by other SMs are read through L2
// (ld.global.cg), never from a stale L1 line.
// --------------------------------------------------------------------------
template <typename T, int D>
__device__ __forceinline__ void merge_heads(const DecodeParams& p, const ItemInfo& it, int64_t item, int qh0,
                                            int nh, int lane) {
  constexpr int HG = 4;                 // heads per pass
  constexpr int VPL = D / 32;           // values per lane (2, 4 or 8)
  constexpr int KU = D == 256 ? 2 : 4;  // splits per load batch
  using Vec = typename std::conditional<VPL == 2, float2, float4>::type;
  constexpr int NV = VPL == 2 ? 1 : VPL / 4;  // vector loads per (head, split)
  constexpr int VW = VPL == 2 ? 2 : 4;        // floats per vector load
  const int ns = it.n_splits;                 // >= 2
  const float2* ml_base = reinterpret_cast<const float2*>(p.ws_ml) + (item * p.hq + qh0) * p.max_splits;

  // (m, l) of splits lane, lane + 32, ... for every head; w0 = weight of split `lane`.
  float w0[HG], m_use[HG], inv_l[HG], lse[HG];
#pragma unroll
  for (int h = 0; h < HG; ++h) {
    const float2* ml = ml_base + (int64_t)h * p.max_splits;
    const bool live = h < nh;
    const float2 first = (live && lane < ns) ? __ldcg(ml + lane) : make_float2(-INFINITY, 0.f);
    float mx = first.x;
    for (int sidx = lane + 32; live && sidx < ns; sidx += 32) mx = fmaxf(mx, __ldcg(ml + sidx).x);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
    m_use[h] = (mx == -INFINITY) ? 0.f : mx;
    w0[h] = (live && lane < ns) ? exp2f(first.x - m_use[h]) : 0.f;
    float l = first.y * w0[h];
    for (int sidx = lane + 32; live && sidx < ns; sidx += 32) {
      const float2 v = __ldcg(ml + sidx);
      l += v.y * exp2f(v.x - m_use[h]);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) l += __shfl_xor_sync(kFull, l, off);
    inv_l[h] = 1.f / l;
    lse[h] = mx * kLn2 + logf(l);
  }

  float acc[HG][VPL];
#pragma unroll
  for (int h = 0; h < HG; ++h)
#pragma unroll
    for (int i = 0; i < VPL; ++i) acc[h][i] = 0.f;
  const float* wo0 = p.ws_o + (item * p.hq + qh0) * p.max_splits * D + lane * VPL;
  const int64_t head_stride = (int64_t)p.max_splits * D;
  for (int s0 = 0; s0 < ns; s0 += 32) {
    float w[HG];
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      if (s0 == 0) {
        w[h] = w0[h];
      } else {
        const bool live = h < nh && s0 + lane < ns;
        w[h] = live ? exp2f(__ldcg(ml_base + (int64_t)h * p.max_splits + s0 + lane).x - m_use[h]) : 0.f;
      }
    }
    const int cnt = min(32, ns - s0);
    for (int k0 = 0; k0 < cnt; k0 += KU) {
      Vec v[KU][HG][NV];
#pragma unroll
      for (int k = 0; k < KU; ++k)
#pragma unroll
        for (int h = 0; h < HG; ++h)
#pragma unroll
          for (int n = 0; n < NV; ++n) {
            const float* src = wo0 + h * head_stride + (int64_t)(s0 + k0 + k) * D + n * 4;
            if (h < nh && k0 + k < cnt) v[k][h][n] = __ldcg(reinterpret_cast<const Vec*>(src));
            else v[k][h][n] = Vec{};
          }
#pragma unroll
      for (int k = 0; k < KU; ++k)
#pragma unroll
        for (int h = 0; h < HG; ++h) {
          const float wk = __shfl_sync(kFull, w[h], (k0 + k) & 31);
#pragma unroll
          for (int n = 0; n < NV; ++n) {
            const float* f = reinterpret_cast<const float*>(&v[k][h][n]);
#pragma unroll
            for (int i = 0; i < VW; ++i) acc[h][n * VW + i] = fmaf(wk, f[i], acc[h][n * VW + i]);
          }
        }
    }
  }
#pragma unroll
  for (int h = 0; h < HG; ++h) {
    if (h >= nh) break;
    T* op = reinterpret_cast<T*>(p.out) + (int64_t)it.qtok * p.o_st + (int64_t)(qh0 + h) * p.o_sh + lane * VPL;
#pragma unroll
    for (int i = 0; i < VPL; ++i) op[i] = Elem<T>::from_float(acc[h][i] * inv_l[h]);
    if (lane == 0) p.lse[(int64_t)it.qtok * p.lse_st + qh0 + h] = lse[h];
  }
}

// Called by every warp after writing its split's partials: the warp that
// completes the (item, kv head) merges all splits of the group. The host clears
// the counters before each launch.
template <typename T, int D>
__device__ __forceinline__ void finish_split(const DecodeParams& p, const ItemInfo& it, int64_t item, int kvh,
                                             int lane) {
  __threadfence();  // this lane's partials are visible device-wide before the arrival
  __syncwarp();
  int prev = 0;
  int32_t* ctr = p.counters + item * p.hkv + kvh;
  if (lane == 0) prev = atomicAdd(ctr, 1);
  prev = __shfl_sync(kFull, prev, 0);
  if (prev != it.n_splits - 1) return;
  __threadfence();
  for (int g0 = 0; g0 < p.group; g0 += 4)
    merge_heads<T, D>(p, it, item, kvh * p.group + g0, min(4, p.group - g0), lane);
}

// --------------------------------------------------------------------------
// Tensor-core path (fp16 / bf16).
// --------------------------------------------------------------------------
// Shared-memory tile of one 16-token block and one kv head: head_dim/64 panels
// of 16 rows x 128 bytes, written by TMA with 128-byte swizzling (16-byte chunk
// c of row r lands at chunk c ^ (r & 7)), so every ldmatrix phase (8 rows, one
// logical chunk) touches 8 distinct bank groups.
template <int D>
struct TmaTile {
  static constexpr int kPanels = D / 64;
  static constexpr int kPanel = 16 * 128;
  static constexpr int kTile = kPanels * kPanel;  // K or V
  static constexpr int kStage = 2 * kTile;        // K then V
};

constexpr int kBarRegion = 1024;  // mbarriers, then the 1 KB-aligned rings

// Threshold (log2 units) by which a block maximum must exceed the running
// reference maximum before O and l are rescaled: probabilities stay <= 2^8.
constexpr float kRescaleThreshold = 8.0f;

template <typename T, int D, int NTH, int STAGES, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
    decode_mma_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v) {
  using Tile = TmaTile<D>;
  constexpr int KS = D / 16;
  extern __shared__ __align__(1024) char smem_raw[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int t = lane & 3;

  int kvh, split;
  const int64_t item = unit_of_warp(p, (int64_t)blockIdx.x * WARPS + warp, kvh, split);
  if (item >= p.num_items || (p.num_items_dev && item >= __ldg(p.num_items_dev))) return;

  const ItemInfo it = item_info(p, (int)item);
  if (split == 0 && kvh == 0) report_item(p, it, lane);
  if (!it.ok) return;
  if (split >= max(it.n_splits, 1)) return;
  const int b0 = split * p.bps;
  const int nb = min(p.bps, it.nblk - b0);  // <= 0 only when the row has no keys
  const BlockIds bids = load_block_ids(p, it, b0, max(nb, 0), lane);

  // Q^T as the B operand (k = head dims, n = heads of the group), kept in registers.
  uint32_t qf[KS][NTH][2];
  {
    const T* qbase = reinterpret_cast<const T*>(p.q) + (int64_t)it.qtok * p.q_st;
#pragma unroll
    for (int nt = 0; nt < NTH; ++nt) {
      const int gh = nt * 8 + g;
      const bool live = gh < p.group;
      const T* qp = qbase + (int64_t)(kvh * p.group + (live ? gh : 0)) * p.q_sh;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        qf[ks][nt][0] = live ? *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 2 * t) : 0u;
        qf[ks][nt][1] = live ? *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 8 + 2 * t) : 0u;
      }
    }
  }

  // 1 KB-aligned layout: [mbarriers (1 KB)] [warp 0 ring] [warp 1 ring] ...
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bar0 = base + warp * STAGES * 8;
  const uint32_t ring = base + kBarRegion + warp * STAGES * Tile::kStage;
  char* ring_ptr = smem_raw + (ring - raw);
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) mbar_init(bar0 + 8 * s, 1);
    fence_mbar_init();
    prefetch_tensor_map(&tmap_k);
    prefetch_tensor_map(&tmap_v);
  }
  __syncwarp();

  // Stage block j (relative to b0) into ring slot j % STAGES (lane 0 issues).
  auto issue = [&](int j) {
    const int bid = bids.get(j);
    if (lane == 0) {
      const int s = j % STAGES;
      const uint32_t bar = bar0 + 8 * s;
      const uint32_t dk = ring + s * Tile::kStage;
      if (bid >= 0) {
        mbar_arrive_expect_tx(bar, Tile::kStage);
#pragma unroll
        for (int pn = 0; pn < Tile::kPanels; ++pn) {
          tma_load_3d(dk + pn * Tile::kPanel, &tmap_k, pn * 64, kvh, bid * 16, bar);
          tma_load_3d(dk + Tile::kTile + pn * Tile::kPanel, &tmap_v, pn * 64, kvh, bid * 16, bar);
        }
      } else {
        mbar_arrive_expect_tx(bar, 0);
      }
    }
  };

  float m_ref[NTH][2], l_part[NTH][2];
  float oacc[KS][NTH][4];
#pragma unroll
  for (int nt = 0; nt < NTH; ++nt) {
    m_ref[nt][0] = m_ref[nt][1] = -INFINITY;
    l_part[nt][0] = l_part[nt][1] = 0.f;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) oacc[mt][nt][0] = oacc[mt][nt][1] = oacc[mt][nt][2] = oacc[mt][nt][3] = 0.f;
  }

  const int npro = min(STAGES, max(nb, 0));
  for (int j = 0; j < npro; ++j) issue(j);

  // Per-lane swizzled offsets. K (ldmatrix, A = keys x dims): row = lane & 15,
  // logical chunk 2*ks + (lane >> 4). V (ldmatrix.trans, A = dims x keys):
  // row = (lane & 7) + 8 * (lane >> 4), logical chunk 2*mt + ((lane >> 3) & 1).
  // Chunk c of a panel row r sits at physical chunk (c & 7) ^ (r & 7).
  const int krow = lane & 15;
  const int khi = lane >> 4;
  const int vrow = (lane & 7) + 8 * (lane >> 4);
  const int vhi = (lane >> 3) & 1;
  uint32_t koff[4], voff[4];
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    koff[m] = krow * 128 + ((((2 * m) | khi) ^ (krow & 7)) << 4);
    voff[m] = vrow * 128 + ((((2 * m) | vhi) ^ (vrow & 7)) << 4);
  }

  bool timed_out = false;
  for (int j = 0; j < nb; ++j) {
    const int s = j % STAGES;
    if (!mbar_wait_bounded(bar0 + 8 * s, (uint32_t)((j / STAGES) & 1))) {
      timed_out = true;
      for (int jj = j + 1; jj < min(j + STAGES, nb); ++jj)
        mbar_wait_bounded(bar0 + 8 * (jj % STAGES), (uint32_t)((jj / STAGES) & 1), 1u << 16);
      break;
    }
    const uint32_t sk = ring + s * Tile::kStage;
    const uint32_t sv = sk + Tile::kTile;
    const int blk = b0 + j;
    const bool bad = bids.get(j) < 0;
    const int real = bad ? 0 : min(16, it.k_len - blk * 16);
    if (real < 16) {
      // V rows of zero-padded or unreadable keys must be exact zeros: the pool
      // past k_len (or an unreadable block) may hold anything, even NaN.
      char* vrows = ring_ptr + (sv - ring);
      for (int c = lane; c < (16 - real) * Tile::kPanels * 8; c += 32) {
        const int row = real + c / (Tile::kPanels * 8);
        const int rem = c % (Tile::kPanels * 8);
        *reinterpret_cast<uint4*>(vrows + (rem >> 3) * Tile::kPanel + row * 128 + (rem & 7) * 16) =
            make_uint4(0u, 0u, 0u, 0u);
      }
      fence_proxy_async_smem();  // order these writes before TMA refills the slot
      __syncwarp();
    }

    // S^T = K Q^T : 16 keys x (8*NTH) heads; two accumulation chains for ILP.
    float sa[NTH][4], sb[NTH][4];
#pragma unroll
    for (int nt = 0; nt < NTH; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) sa[nt][c] = sb[nt][c] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4(sk + (ks >> 2) * Tile::kPanel + koff[ks & 3], a0, a1, a2, a3);
#pragma unroll
      for (int nt = 0; nt < NTH; ++nt) {
        if (ks & 1) Mma<T>::run(sb[nt], a0, a1, a2, a3, qf[ks][nt][0], qf[ks][nt][1]);
        else Mma<T>::run(sa[nt], a0, a1, a2, a3, qf[ks][nt][0], qf[ks][nt][1]);
      }
    }

    // Scale into the log2 domain and mask (keys past the visible range: -inf;
    // zero-padded keys of the last block inside it: score 0).
    const int key0 = blk * 16 + g;
    float x[NTH][4];
#pragma unroll
    for (int nt = 0; nt < NTH; ++nt)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int key = key0 + (c >> 1) * 8;
        float v = (sa[nt][c] + sb[nt][c]) * p.scale_log2;
        if (bad || key >= it.n_vis) v = -INFINITY;
        else if (key >= it.k_len) v = 0.f;
        x[nt][c] = v;
      }

    // Online softmax per head column with a lazily updated reference max.
    float mb[NTH][2];
    bool need = false;
#pragma unroll
    for (int nt = 0; nt < NTH; ++nt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v = fmaxf(x[nt][h], x[nt][h + 2]);
        v = fmaxf(v, __shfl_xor_sync(kFull, v, 4));
        v = fmaxf(v, __shfl_xor_sync(kFull, v, 8));
        v = fmaxf(v, __shfl_xor_sync(kFull, v, 16));
        mb[nt][h] = v;
        need |= v > m_ref[nt][h] + kRescaleThreshold;
      }
    if (__any_sync(kFull, need)) {
      float corr[NTH][2];
#pragma unroll
      for (int nt = 0; nt < NTH; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (mb[nt][h] > m_ref[nt][h] + kRescaleThreshold) {
            corr[nt][h] = exp2f(m_ref[nt][h] - mb[nt][h]);  // 0 when m_ref is -inf
            m_ref[nt][h] = mb[nt][h];
          } else {
            corr[nt][h] = 1.f;
          }
          l_part[nt][h] *= corr[nt][h];
        }
#pragma unroll
      for (int mt = 0; mt < KS; ++mt)
#pragma unroll
        for (int nt = 0; nt < NTH; ++nt) {
          oacc[mt][nt][0] *= corr[nt][0];
          oacc[mt][nt][1] *= corr[nt][1];
          oacc[mt][nt][2] *= corr[nt][0];
          oacc[mt][nt][3] *= corr[nt][1];
        }
    }
#pragma unroll
    for (int nt = 0; nt < NTH; ++nt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float m_use = m_ref[nt][h] == -INFINITY ? 0.f : m_ref[nt][h];
        x[nt][h] = exp2f(x[nt][h] - m_use);
        x[nt][h + 2] = exp2f(x[nt][h + 2] - m_use);
        l_part[nt][h] += x[nt][h] + x[nt][h + 2];
      }

    // P^T (k = keys, n = heads) operand fragments. P is split into a 16-bit
    // high part and the 16-bit rounding of its remainder, so P V is exact to
    // ~2^-17 relative instead of carrying the 2^-9 error of one bf16 rounding.
    uint32_t pb0[NTH], pb1[NTH], pl0[NTH], pl1[NTH];
#pragma unroll
    for (int nt = 0; nt < NTH; ++nt) {
      const uint32_t h0 = Mma<T>::pack(x[nt][0], x[nt][1]);
      const uint32_t h1 = Mma<T>::pack(x[nt][2], x[nt][3]);
      const float2 f0 = Mma<T>::unpack(h0);
      const float2 f1 = Mma<T>::unpack(h1);
      pb0[nt] = movmatrix_trans(h0);
      pb1[nt] = movmatrix_trans(h1);
      pl0[nt] = movmatrix_trans(Mma<T>::pack(x[nt][0] - f0.x, x[nt][1] - f0.y));
      pl1[nt] = movmatrix_trans(Mma<T>::pack(x[nt][2] - f1.x, x[nt][3] - f1.y));
    }

    // O^T += V^T P^T : head_dim x heads.
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4_trans(sv + (mt >> 2) * Tile::kPanel + voff[mt & 3], a0, a1, a2, a3);
#pragma unroll
      for (int nt = 0; nt < NTH; ++nt) {
        Mma<T>::run(oacc[mt][nt], a0, a1, a2, a3, pb0[nt], pb1[nt]);
        Mma<T>::run(oacc[mt][nt], a0, a1, a2, a3, pl0[nt], pl1[nt]);
      }
    }
    __syncwarp();
    if (j + STAGES < nb) issue(j + STAGES);
  }
  // A timed-out warp still reports its (invalid) partial so the split counter
  // of its item stays consistent; the error word flags the call.
  if (timed_out && lane == 0) atomic_or_err(p.err, SEB_ERRBIT_TIMEOUT);

  float l_tot[NTH][2];
#pragma unroll
  for (int nt = 0; nt < NTH; ++nt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float l = l_part[nt][h];
      l += __shfl_xor_sync(kFull, l, 4);
      l += __shfl_xor_sync(kFull, l, 8);
      l += __shfl_xor_sync(kFull, l, 16);
      l_tot[nt][h] = l;
    }

  if (it.n_splits <= 1) {
    T* obase = reinterpret_cast<T*>(p.out) + (int64_t)it.qtok * p.o_st;
#pragma unroll
    for (int nt = 0; nt < NTH; ++nt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int gh = nt * 8 + 2 * t + h;
        if (gh >= p.group) continue;
        const int qh = kvh * p.group + gh;
        T* op = obase + (int64_t)qh * p.o_sh;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          op[mt * 16 + g] = Elem<T>::from_float(oacc[mt][nt][h] / l_tot[nt][h]);
          op[mt * 16 + g + 8] = Elem<T>::from_float(oacc[mt][nt][h + 2] / l_tot[nt][h]);
        }
        if (g == 0) p.lse[(int64_t)it.qtok * p.lse_st + qh] = m_ref[nt][h] * kLn2 + logf(l_tot[nt][h]);
      }
  } else {
#pragma unroll
    for (int nt = 0; nt < NTH; ++nt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int gh = nt * 8 + 2 * t + h;
        if (gh >= p.group) continue;
        const int qh = kvh * p.group + gh;
        const int64_t slot = ((item * p.hq + qh) * p.max_splits + split);
        float* wo = p.ws_o + slot * D;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          wo[mt * 16 + g] = oacc[mt][nt][h];
          wo[mt * 16 + g + 8] = oacc[mt][nt][h + 2];
        }
        if (g == 0) {
          p.ws_ml[slot * 2] = m_ref[nt][h];
          p.ws_ml[slot * 2 + 1] = l_tot[nt][h];
        }
      }
    finish_split<T, D>(p, it, item, kvh, lane);
  }
}

// --------------------------------------------------------------------------
// CUDA-core path (fp32, or shapes without a tensor-core kernel). Same work
// decomposition; each lane owns head dims lane + 32*i; keys are visited one at
// a time with a full-warp dot-product reduction.
// --------------------------------------------------------------------------
template <typename T, int D, int GMAX, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) decode_simt_kernel(const DecodeParams p) {
  constexpr int DL = D / 32;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int kvh, split;
  const int64_t item = unit_of_warp(p, (int64_t)blockIdx.x * WARPS + warp, kvh, split);
  if (item >= p.num_items || (p.num_items_dev && item >= __ldg(p.num_items_dev))) return;
  const ItemInfo it = item_info(p, (int)item);
  if (split == 0 && kvh == 0) report_item(p, it, lane);
  if (!it.ok) return;
  if (split >= max(it.n_splits, 1)) return;
  const int b0 = split * p.bps;
  const int nb = min(p.bps, it.nblk - b0);
  const BlockIds bids = load_block_ids(p, it, b0, max(nb, 0), lane);

  float qv[GMAX][DL];
  const T* qbase = reinterpret_cast<const T*>(p.q) + (int64_t)it.qtok * p.q_st;
#pragma unroll
  for (int gh = 0; gh < GMAX; ++gh)
#pragma unroll
    for (int i = 0; i < DL; ++i)
      qv[gh][i] = gh < p.group
                      ? Elem<T>::to_float(qbase[(int64_t)(kvh * p.group + gh) * p.q_sh + lane + 32 * i])
                      : 0.f;

  float m[GMAX], l[GMAX], o[GMAX][DL];
#pragma unroll
  for (int gh = 0; gh < GMAX; ++gh) {
    m[gh] = -INFINITY;
    l[gh] = 0.f;
#pragma unroll
    for (int i = 0; i < DL; ++i) o[gh][i] = 0.f;
  }

  const T* kc = reinterpret_cast<const T*>(p.k_cache);
  const T* vc = reinterpret_cast<const T*>(p.v_cache);
  for (int j = 0; j < nb; ++j) {
    const int blk = b0 + j;
    const int bid = bids.get(j);
    const int vis = min(16, it.n_vis - blk * 16);
    const int real = bid >= 0 ? min(vis, it.k_len - blk * 16) : 0;
    for (int r = 0; r < vis; ++r) {
      float kv[DL], vv[DL];
      if (r < real) {
        const int64_t off = (((int64_t)bid * 16 + r) * p.hkv + kvh) * D + lane;
#pragma unroll
        for (int i = 0; i < DL; ++i) {
          kv[i] = Elem<T>::to_float(kc[off + 32 * i]);
          vv[i] = Elem<T>::to_float(vc[off + 32 * i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < DL; ++i) kv[i] = vv[i] = 0.f;
      }
      const bool readable = (r < real) || (bid >= 0);
#pragma unroll
      for (int gh = 0; gh < GMAX; ++gh) {
        if (gh >= p.group) break;
        float sdot = 0.f;
#pragma unroll
        for (int i = 0; i < DL; ++i) sdot = fmaf(qv[gh][i], kv[i], sdot);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) sdot += __shfl_xor_sync(kFull, sdot, off);
        // unreadable block (bad id): treated as masked
        const float x = readable ? sdot * p.scale_log2 : -INFINITY;
        const float m_new = fmaxf(m[gh], x);
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        const float cr = exp2f(m[gh] - m_use);
        const float pr = exp2f(x - m_use);
        l[gh] = l[gh] * cr + pr;
#pragma unroll
        for (int i = 0; i < DL; ++i) o[gh][i] = fmaf(pr, vv[i], o[gh][i] * cr);
        m[gh] = m_new;
      }
    }
  }

  if (it.n_splits <= 1) {
    T* obase = reinterpret_cast<T*>(p.out) + (int64_t)it.qtok * p.o_st;
#pragma unroll
    for (int gh = 0; gh < GMAX; ++gh) {
      if (gh >= p.group) break;
      const int qh = kvh * p.group + gh;
#pragma unroll
      for (int i = 0; i < DL; ++i)
        obase[(int64_t)qh * p.o_sh + lane + 32 * i] = Elem<T>::from_float(o[gh][i] / l[gh]);
      if (lane == 0) p.lse[(int64_t)it.qtok * p.lse_st + qh] = m[gh] * kLn2 + logf(l[gh]);
    }
  } else {
#pragma unroll
    for (int gh = 0; gh < GMAX; ++gh) {
      if (gh >= p.group) break;
      const int qh = kvh * p.group + gh;
      const int64_t slot = ((item * p.hq + qh) * p.max_splits + split);
#pragma unroll
      for (int i = 0; i < DL; ++i) p.ws_o[slot * D + lane + 32 * i] = o[gh][i];
      if (lane == 0) {
        p.ws_ml[slot * 2] = m[gh];
        p.ws_ml[slot * 2 + 1] = l[gh];
      }
    }
    finish_split<T, D>(p, it, item, kvh, lane);
  }
}

// ------------------------------------------------------------------ launching
// Warps per CTA (each its own work item) and ring depth per warp. Shared memory
// per CTA = 2 KB + warps * stages * 32 * head_dim bytes.
#ifndef SEB_DECODE_WARPS
#define SEB_DECODE_WARPS 4
#endif
#ifndef SEB_DECODE_STAGES
#define SEB_DECODE_STAGES 2
#endif
constexpr int kMmaWarps = SEB_DECODE_WARPS;
constexpr int kMmaStages = SEB_DECODE_STAGES;
template <int D>
constexpr int mma_stages() {
  // keep the D = 256 ring within the 227 KB a CTA may use
  return (kMmaWarps * kMmaStages * TmaTile<D>::kStage + 3 * 1024 <= 227 * 1024)
             ? kMmaStages
             : (227 * 1024 - 3 * 1024) / (kMmaWarps * TmaTile<D>::kStage);
}
constexpr int kSimtWarps = 4;

// Bytes of the split counters at the end of the decode workspace.
int64_t counter_bytes(int64_t num_items, int64_t hkv) { return ((num_items * hkv * 4 + 15) / 16) * 16; }

// Longest split the automatic rule picks. Measured over 200 calls: config 2
// (64 rows, k_len U[1024, 8192], head_dim 128) 221.5 / 217.9 / 217.0 us at 32 /
// 40 / 64 blocks; config-4 decode rows (256 rows, lognormal lengths, head_dim
// 64, a 264-block table) 78.7 / 74.5 / 84.1 us: longer splits cut the merges
// and the idle CTAs of a wide table, but past about 40 blocks a short batch's
// last splits run alone.
constexpr int kAutoMaxBps = 40;

int choose_bps(int num_items, int hkv, int64_t max_blocks, int requested) {
  if (requested > 0) return requested > kMaxBps ? kMaxBps : requested;
  // Aim for about two waves of 12 resident warps per SM, assuming rows fill
  // about half of the block-table width; long splits (up to kAutoMaxBps blocks)
  // keep the partial-result traffic small, >= 8 blocks keep the copy ring busy.
  const double est_blocks = 0.5 * (double)num_items * hkv * (double)max_blocks;
  const double slots = (double)num_sms() * 12.0 * 2.0;
  int bps = (int)std::ceil(est_blocks / slots);
  if (bps < 8) bps = 8;
  if (bps > kAutoMaxBps) bps = kAutoMaxBps;
  return bps;
}

template <typename T, int D, int NTH>
int launch_mma(const DecodeParams& p, int64_t n_warps, cudaStream_t s) {
  constexpr int stages = mma_stages<D>();
  constexpr int smem = 1024 /* alignment slack */ + kBarRegion + kMmaWarps * stages * TmaTile<D>::kStage;
  static_assert(kMmaWarps * stages * 8 <= kBarRegion, "mbarrier region too small");
  constexpr auto kern = decode_mma_kernel<T, D, NTH, stages, kMmaWarps>;
  int rc = set_smem_limit_once<kern>(smem);
  if (rc != SEB_OK) return rc;
  CUtensorMap tk, tv;
  const int dtype = std::is_same<T, __nv_bfloat16>::value ? SEB_BF16 : SEB_F16;
  rc = kv_tensor_map(&tk, p.k_cache, dtype, p.num_blocks, p.hkv, D);
  if (rc != SEB_OK) return rc;
  rc = kv_tensor_map(&tv, p.v_cache, dtype, p.num_blocks, p.hkv, D);
  if (rc != SEB_OK) return rc;
  const int64_t grid = (n_warps + kMmaWarps - 1) / kMmaWarps;
  kern<<<(unsigned)grid, kMmaWarps * 32, smem, s>>>(p, tk, tv);
  return launch_status("decode_mma_kernel");
}

template <typename T, int D, int GMAX>
int launch_simt(const DecodeParams& p, int64_t n_warps, cudaStream_t s) {
  const int64_t grid = (n_warps + kSimtWarps - 1) / kSimtWarps;
  decode_simt_kernel<T, D, GMAX, kSimtWarps><<<(unsigned)grid, kSimtWarps * 32, 0, s>>>(p);
  return launch_status("decode_simt_kernel");
}

template <typename T, int D>
int launch_simt_g(const DecodeParams& p, int64_t n_warps, cudaStream_t s) {
  if (p.group <= 1) return launch_simt<T, D, 1>(p, n_warps, s);
  if (p.group <= 2) return launch_simt<T, D, 2>(p, n_warps, s);
  if (p.group <= 4) return launch_simt<T, D, 4>(p, n_warps, s);
  if (p.group <= 8) return launch_simt<T, D, 8>(p, n_warps, s);
  return launch_simt<T, D, 16>(p, n_warps, s);
}

template <typename T, int D>
int launch_typed(const DecodeParams& p, int64_t n_warps, bool tensor_core, cudaStream_t s) {
  int rc;
  if constexpr (sizeof(T) == 2) {
    if (tensor_core) {
      rc = p.group <= 8 ? launch_mma<T, D, 1>(p, n_warps, s) : launch_mma<T, D, 2>(p, n_warps, s);
    } else {
      rc = launch_simt_g<T, D>(p, n_warps, s);
    }
  } else {
    rc = launch_simt_g<T, D>(p, n_warps, s);
  }
  return rc;
}

template <typename T>
int launch_dim(const DecodeParams& p, int D, int64_t n_warps, bool tc, cudaStream_t s) {
  switch (D) {
    case 64: return launch_typed<T, 64>(p, n_warps, tc, s);
    case 128: return launch_typed<T, 128>(p, n_warps, tc, s);
    case 256: return launch_typed<T, 256>(p, n_warps, tc, s);
    default: set_error("head_dim %d not supported (64, 128, 256)", D); return SEB_EUNSUPPORTED;
  }
}

}  // namespace
}  // namespace seb

extern "C" int64_t seb_paged_decode_workspace_size(int32_t num_items, int32_t num_q_heads,
                                                   int32_t num_kv_heads, int32_t head_dim,
                                                   int64_t max_blocks, int32_t blocks_per_split) {
  using namespace seb;
  if (num_items <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_blocks <= 0)
    return 0;
  const int bps = choose_bps(num_items, num_kv_heads, max_blocks, blocks_per_split);
  const int64_t max_splits = (max_blocks + bps - 1) / bps;
  if (max_splits <= 1) return 0;
  return (int64_t)num_items * num_q_heads * max_splits * (head_dim + 2) * (int64_t)sizeof(float) +
         seb::counter_bytes(num_items, num_kv_heads);
}

namespace seb {

int paged_decode_impl(const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* k_cache,
                      const void* v_cache, int64_t num_blocks, const int32_t* block_table, int64_t block_table_stride,
                      int64_t max_blocks, const int32_t* q_starts, const int32_t* k_lens, const int32_t* q_pos_offsets,
                      int32_t num_rows, int32_t total_query, const int32_t* item_query, const int32_t* item_row,
                      int32_t num_items, const int32_t* num_items_dev, int32_t num_q_heads, int32_t num_kv_heads,
                      int32_t head_dim, int32_t dtype, float scale, int32_t is_causal, int32_t blocks_per_split,
                      void* out, int64_t out_stride_token, int64_t out_stride_head, float* lse,
                      int64_t lse_stride_token, void* workspace, int64_t workspace_bytes, int32_t* err,
                      void* stream) {
  const int es = elem_size(dtype);
  SEB_CHECK_ARG(es > 0, "seb_paged_decode: unknown dtype %d", dtype);
  SEB_CHECK_ARG(num_items >= 0 && num_rows >= 0 && total_query >= 0, "seb_paged_decode: negative count");
  if (num_items == 0) return SEB_OK;
  SEB_CHECK_ARG(num_rows > 0, "seb_paged_decode: items given but no rows");
  SEB_CHECK_ARG(num_q_heads > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
                "seb_paged_decode: num_q_heads (%d) must be a positive multiple of num_kv_heads (%d)",
                num_q_heads, num_kv_heads);
  const int group = num_q_heads / num_kv_heads;
  SEB_CHECK_ARG(group <= 16, "seb_paged_decode: GQA group %d > 16 not supported", group);
  SEB_CHECK_ARG(q && k_cache && v_cache && block_table && q_starts && k_lens && q_pos_offsets && out && lse,
                "seb_paged_decode: NULL pointer argument");
  SEB_CHECK_ARG(num_blocks > 0 && max_blocks > 0 && block_table_stride >= max_blocks,
                "seb_paged_decode: bad block table shape (num_blocks %lld, max_blocks %lld, stride %lld)",
                (long long)num_blocks, (long long)max_blocks, (long long)block_table_stride);
  SEB_CHECK_ARG(aligned(k_cache, 16) && aligned(v_cache, 16), "seb_paged_decode: KV pool not 16-byte aligned");
  const bool tc = (dtype != SEB_F32);
  if (tc) {
    SEB_CHECK_ARG(aligned(q, 4) && q_stride_token % 2 == 0 && q_stride_head % 2 == 0,
                  "seb_paged_decode: q must be 4-byte aligned with even strides");
  }

  DecodeParams p;
  p.q = static_cast<const char*>(q);
  p.q_st = q_stride_token;
  p.q_sh = q_stride_head;
  p.k_cache = static_cast<const char*>(k_cache);
  p.v_cache = static_cast<const char*>(v_cache);
  p.num_blocks = num_blocks;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.max_blocks = max_blocks;
  p.q_starts = q_starts;
  p.k_lens = k_lens;
  p.q_pos = q_pos_offsets;
  p.num_rows = num_rows;
  p.total_query = total_query;
  p.item_query = item_query;
  p.item_row = item_row;
  p.num_items = num_items;
  p.num_items_dev = num_items_dev;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.group = group;
  p.scale_log2 = scale * kLog2e;
  p.causal = is_causal ? 1 : 0;
  p.bps = choose_bps(num_items, num_kv_heads, max_blocks, blocks_per_split);
  p.max_splits = (int)((max_blocks + p.bps - 1) / p.bps);
  p.out = static_cast<char*>(out);
  p.o_st = out_stride_token;
  p.o_sh = out_stride_head;
  p.lse = lse;
  p.lse_st = lse_stride_token;
  p.err = err;
  p.ws_o = nullptr;
  p.ws_ml = nullptr;
  p.counters = nullptr;
  if (p.max_splits > 1) {
    const int64_t need = seb_paged_decode_workspace_size(num_items, num_q_heads, num_kv_heads, head_dim,
                                                         max_blocks, blocks_per_split);
    if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 16)) {
      set_error("seb_paged_decode: workspace of %lld bytes (16-byte aligned) required, got %lld",
                (long long)need, (long long)workspace_bytes);
      return SEB_EWORKSPACE;
    }
    p.ws_o = static_cast<float*>(workspace);
    p.ws_ml = p.ws_o + (int64_t)num_items * num_q_heads * p.max_splits * head_dim;
    p.counters = reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + need -
                                            counter_bytes(num_items, num_kv_heads));
  }
  const int64_t n_warps = (int64_t)num_items * num_kv_heads * p.max_splits;
  SEB_CHECK_ARG((n_warps + 3) / 4 < (1ll << 31), "seb_paged_decode: grid too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p.counters)
    SEB_CHECK_CUDA(cudaMemsetAsync(p.counters, 0, (size_t)counter_bytes(num_items, num_kv_heads), s));
  switch (dtype) {
    case SEB_BF16: return launch_dim<__nv_bfloat16>(p, head_dim, n_warps, tc, s);
    case SEB_F16: return launch_dim<__half>(p, head_dim, n_warps, tc, s);
    default: return launch_dim<float>(p, head_dim, n_warps, false, s);
  }
}

}  // namespace seb

extern "C" int seb_paged_decode(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                                const void* k_cache, const void* v_cache, int64_t num_blocks,
                                const int32_t* block_table, int64_t block_table_stride,
                                int64_t max_blocks, const int32_t* q_starts, const int32_t* k_lens,
                                const int32_t* q_pos_offsets, int32_t num_rows, int32_t total_query,
                                const int32_t* item_query, const int32_t* item_row,
                                int32_t num_items, int32_t num_q_heads, int32_t num_kv_heads,
                                int32_t head_dim, int32_t dtype, float scale, int32_t is_causal,
                                int32_t blocks_per_split, void* out, int64_t out_stride_token,
                                int64_t out_stride_head, float* lse, int64_t lse_stride_token,
                                void* workspace, int64_t workspace_bytes, int32_t* err,
                                void* stream) {
  seb::clear_error();
  return seb::paged_decode_impl(q, q_stride_token, q_stride_head, k_cache, v_cache, num_blocks, block_table,
                                block_table_stride, max_blocks, q_starts, k_lens, q_pos_offsets, num_rows,
                                total_query, item_query, item_row, num_items, nullptr, num_q_heads, num_kv_heads,
                                head_dim, dtype, scale, is_causal, blocks_per_split, out, out_stride_token,
                                out_stride_head, lse, lse_stride_token, workspace, workspace_bytes, err, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of seb_paged_decode.
//
// Its split-K scratch is this file-scope device array, so the call needs no
// workspace from the caller and performs no device allocation. The array is
// part of the library image: every GPU that loads the library holds
// SEB_NOALLOC_SCRATCH_BYTES of it until the process exits. In host code the
// symbol is only a host-side stand-in, so the device address is looked up with
// cudaGetSymbolAddress once per device (with that device current) and cached.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[SEB_NOALLOC_SCRATCH_BYTES];

namespace seb {
namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device.
int noalloc_scratch_address(void** out) {
  int dev = -1;
  SEB_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("seb_paged_decode_noalloc: device ordinal %d outside [0, %d)", dev, kMaxDevices);
    return SEB_EINVAL;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("seb_paged_decode_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(e));
      return SEB_ECUDA;
    }
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return SEB_OK;
}

}  // namespace
}  // namespace seb

extern "C" int seb_paged_decode_noalloc(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                                        const void* k_cache, const void* v_cache, int64_t num_blocks,
                                        const int32_t* block_table, int64_t block_table_stride,
                                        int64_t max_blocks, const int32_t* q_starts, const int32_t* k_lens,
                                        const int32_t* q_pos_offsets, int32_t num_rows, int32_t total_query,
                                        const int32_t* item_query, const int32_t* item_row, int32_t num_items,
                                        int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                        int32_t dtype, float scale, int32_t is_causal, int32_t blocks_per_split,
                                        void* out, int64_t out_stride_token, int64_t out_stride_head,
                                        float* lse, int64_t lse_stride_token, int32_t* err, void* stream) {
  using namespace seb;
  clear_error();
  const int64_t need = seb_paged_decode_workspace_size(num_items, num_q_heads, num_kv_heads, head_dim, max_blocks,
                                                       blocks_per_split);
  if (need > (int64_t)SEB_NOALLOC_SCRATCH_BYTES) {
    // The smallest need any blocks_per_split reaches is the one at the cap of
    // kMaxBps blocks per split; past it only a smaller batch helps.
    const int64_t floor_need = seb_paged_decode_workspace_size(num_items, num_q_heads, num_kv_heads, head_dim,
                                                               max_blocks, kMaxBps);
    set_error("seb_paged_decode_noalloc: this call needs %lld bytes of split-K scratch but the built-in scratch "
              "holds %lld bytes; blocks_per_split is capped at %d, where this batch still needs %lld bytes: "
              "split the batch, or call seb_paged_decode with a workspace",
              (long long)need, (long long)SEB_NOALLOC_SCRATCH_BYTES, kMaxBps, (long long)floor_need);
    return SEB_EWORKSPACE;
  }
  // A call that needs no scratch (no items, or every row fits one split) never
  // looks the array up, so only calls that use it carry the first-call rule.
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = noalloc_scratch_address(&scratch);
    if (rc != SEB_OK) return rc;
  }
  return seb_paged_decode(q, q_stride_token, q_stride_head, k_cache, v_cache, num_blocks, block_table,
                          block_table_stride, max_blocks, q_starts, k_lens, q_pos_offsets, num_rows, total_query,
                          item_query, item_row, num_items, num_q_heads, num_kv_heads, head_dim, dtype, scale,
                          is_causal, blocks_per_split, out, out_stride_token, out_stride_head, lse,
                          lse_stride_token, scratch, need > 0 ? (int64_t)SEB_NOALLOC_SCRATCH_BYTES : 0, err,
                          stream);
}
