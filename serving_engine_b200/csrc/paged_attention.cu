// One call for a whole mixed batch described by the reference's own step
// metadata: the rows' q_lens / k_lens / q_starts / q_pos_offsets and the padded
// block table that build_paged_batch_metadata (serving_engine/
// paged_attention_kernel.py:163-200) returns, with no host-side knowledge of
// which rows decode and which prefill.
//
// A one-CTA routing kernel reads q_lens on the device and writes, into the
// caller's workspace, the decode items (q_len == 1 rows: token, row) and the
// prefill work units (q_len > 1 rows x kv heads x pairs of 128-row Q tiles)
// with their counts. The split-K decode kernel then runs over the decode items
// and the tcgen05 prefill kernel over the unit list; each is launched with a
// grid sized from host-known bounds (rows, total_query) and reads the real
// count from the device, so surplus warps / clusters exit at once and the host
// never reads a device value back.
#include "seb_common.cuh"

#include <algorithm>

namespace seb {
namespace {

constexpr int kRouteThreads = 1024;

struct RouteParams {
  const int32_t* q_lens;
  const int32_t* k_lens;
  const int32_t* q_starts;
  int32_t num_rows;
  int64_t max_blocks;
  int32_t hkv;
  int32_t pair_queries;  // queries per pair of Q tiles: 2 * (128 / group)
  int32_t unit_cap;
  int32_t* counts;       // [0] decode items, [1] prefill units
  int32_t* dec_tokens;   // [num_rows]
  int32_t* dec_rows;     // [num_rows]
  int32_t* units;        // [2 * unit_cap]
  int32_t* err;
};

// Exclusive scan of v over the CTA's 1024 threads; returns this thread's offset
// and writes the total to *total (every thread sees it after the call).
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
    int incl = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    warp_sums[lane] = incl - w;  // exclusive warp offsets
    if (lane == 31) *total = incl;
  }
  __syncthreads();
  const int off = warp_sums[warp] + x - v;
  __syncthreads();  // warp_sums is reused by the next scan
  return off;
}

// Rows in order; decode items keep the rows' order, and each prefill row's units
// are its kv heads, each with its Q-tile pairs latest first (they see the most
// keys), the order the prefill kernel's own row x kv head x pair grid uses. The
// scans give each row its place; one warp per row then writes the row's units
// (a 4,096-token row at head_dim 64 has 512 of them), 32 lanes at a time.
__global__ void __launch_bounds__(kRouteThreads) route_rows_kernel(const RouteParams r) {
  __shared__ int warp_sums[32];
  __shared__ int totals[2];
  __shared__ int s_off[kRouteThreads], s_n[kRouteThreads], s_mp[kRouteThreads];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int dec_base = 0, unit_base = 0;
  for (int r0 = 0; r0 < r.num_rows; r0 += kRouteThreads) {
    const int row = r0 + threadIdx.x;
    int is_dec = 0, nunits = 0, mp = 0, q_start = 0;
    if (row < r.num_rows) {
      const int q_len = __ldg(r.q_lens + row);
      const int k_len = __ldg(r.k_lens + row);
      q_start = __ldg(r.q_starts + row);
      if (q_len > 0 && (int64_t)((max(k_len, 0) + 15) >> 4) > r.max_blocks) atomic_or_err(r.err, SEB_ERRBIT_KLEN);
      if (q_len == 1) {
        is_dec = 1;
      } else if (q_len > 1) {
        mp = (q_len + r.pair_queries - 1) / r.pair_queries;
        nunits = r.hkv * mp;
      }
    }
    const int dec_off = block_exclusive_scan(is_dec, warp_sums, &totals[0]) + dec_base;
    const int unit_off = block_exclusive_scan(nunits, warp_sums, &totals[1]) + unit_base;
    if (is_dec) {
      r.dec_tokens[dec_off] = q_start;
      r.dec_rows[dec_off] = row;
    }
    s_off[threadIdx.x] = unit_off;
    s_n[threadIdx.x] = nunits;
    s_mp[threadIdx.x] = mp;
    __syncthreads();
    const int chunk_rows = min(kRouteThreads, r.num_rows - r0);
    for (int i = warp; i < chunk_rows; i += kRouteThreads / 32) {
      const int n = s_n[i], off = s_off[i], m = s_mp[i];
      for (int k = lane; k < n; k += 32) {
        const int u = off + k;
        if (u >= r.unit_cap) {  // cannot happen with the host's bound; never write past the list
          atomic_or_err(r.err, SEB_ERRBIT_META);
          break;
        }
        const int kvh = k / m;
        const int pr = m - 1 - (k % m);
        r.units[2 * u] = r0 + i;
        r.units[2 * u + 1] = (pr << 8) | kvh;
      }
    }
    dec_base += totals[0];
    unit_base += totals[1];
    __syncthreads();  // totals and the row arrays are rewritten by the next chunk
  }
  if (threadIdx.x == 0) {
    r.counts[0] = dec_base;
    r.counts[1] = min(unit_base, r.unit_cap);
  }
}

bool prefill_shape_ok(int dtype, int head_dim, int group) {
  return (dtype == SEB_BF16 || dtype == SEB_F16) && (head_dim == 64 || head_dim == 128) &&
         (group == 1 || group == 2 || group == 4 || group == 8 || group == 16);
}

bool prefill_layout_ok(const void* q, int64_t q_st, int64_t q_sh, const void* out, int64_t o_st, int64_t o_sh,
                       int head_dim, int hq) {
  return aligned(q, 16) && q_st % 8 == 0 && q_sh % 8 == 0 && q_sh >= head_dim && q_st >= q_sh * hq &&
         aligned(out, 16) && o_st % 8 == 0 && o_sh % 8 == 0;
}

// Upper bound on the prefill units of any batch with these host-known sizes:
// sum over prefill rows of hkv * ceil(q_len / pair_queries), where the rows
// have q_len >= 2 and sum to at most total_query tokens.
int64_t unit_bound(int64_t num_rows, int64_t total_query, int hkv, int pair_queries) {
  const int64_t n_pre = std::min<int64_t>(num_rows, total_query / 2);
  return (int64_t)hkv * (total_query / pair_queries + n_pre);
}

struct RouteLayout {
  int64_t counts, dec_tokens, dec_rows, units, bytes;
};

RouteLayout route_layout(int64_t num_rows, int64_t unit_cap) {
  RouteLayout l;
  l.counts = 0;
  l.dec_tokens = 16;
  l.dec_rows = l.dec_tokens + 4 * num_rows;
  l.units = l.dec_rows + 4 * num_rows;
  l.bytes = ((l.units + 8 * unit_cap) + 255) / 256 * 256;
  return l;
}

}  // namespace
}  // namespace seb

extern "C" int64_t seb_paged_attention_workspace_size(int32_t num_rows, int32_t total_query, int32_t num_q_heads,
                                                      int32_t num_kv_heads, int32_t head_dim, int64_t max_blocks) {
  using namespace seb;
  if (num_rows <= 0 || total_query <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 ||
      num_q_heads % num_kv_heads != 0 || head_dim <= 0 || max_blocks <= 0)
    return 0;
  const int group = num_q_heads / num_kv_heads;
  const int pair_queries = 2 * std::max(1, 128 / group);
  const int64_t cap = unit_bound(num_rows, total_query, num_kv_heads, pair_queries);
  const int64_t decode = seb_paged_decode_workspace_size(std::max(num_rows, total_query), num_q_heads,
                                                         num_kv_heads, head_dim, max_blocks, 0);
  return route_layout(num_rows, cap).bytes + decode;
}

extern "C" int seb_paged_attention(const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* k_cache,
                                   const void* v_cache, int64_t num_blocks, const int32_t* block_table,
                                   int64_t block_table_stride, int64_t max_blocks, const int32_t* q_lens,
                                   const int32_t* k_lens, const int32_t* q_starts, const int32_t* q_pos_offsets,
                                   int32_t num_rows, int32_t total_query, int32_t num_q_heads, int32_t num_kv_heads,
                                   int32_t head_dim, int32_t dtype, float scale, int32_t is_causal, void* out,
                                   int64_t out_stride_token, int64_t out_stride_head, float* lse,
                                   int64_t lse_stride_token, void* workspace, int64_t workspace_bytes, int32_t* err,
                                   void* stream) {
  using namespace seb;
  clear_error();
  SEB_CHECK_ARG(num_rows >= 0 && total_query >= 0, "seb_paged_attention: negative count");
  if (num_rows == 0 || total_query == 0) return SEB_OK;
  SEB_CHECK_ARG(q_lens && k_lens && q_starts && q_pos_offsets && block_table,
                "seb_paged_attention: NULL metadata pointer");
  SEB_CHECK_ARG(num_q_heads > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
                "seb_paged_attention: num_q_heads (%d) must be a positive multiple of num_kv_heads (%d)",
                num_q_heads, num_kv_heads);
  SEB_CHECK_ARG(max_blocks > 0, "seb_paged_attention: empty block table");
  const int64_t need = seb_paged_attention_workspace_size(num_rows, total_query, num_q_heads, num_kv_heads,
                                                          head_dim, max_blocks);
  if (workspace == nullptr || workspace_bytes < need || !aligned(workspace, 256)) {
    set_error("seb_paged_attention: workspace of %lld bytes (256-byte aligned) required, got %lld",
              (long long)need, (long long)workspace_bytes);
    return SEB_EWORKSPACE;
  }
  const int group = num_q_heads / num_kv_heads;
  const bool route = total_query > num_rows && prefill_shape_ok(dtype, head_dim, group) &&
                     prefill_layout_ok(q, q_stride_token, q_stride_head, out, out_stride_token, out_stride_head,
                                       head_dim, num_q_heads);
  if (!route) {
    // Every token through the split-K kernel (rows found by binary search): the
    // batch is all decode rows, or its shape has no tcgen05 prefill kernel.
    return paged_decode_impl(q, q_stride_token, q_stride_head, k_cache, v_cache, num_blocks, block_table,
                             block_table_stride, max_blocks, q_starts, k_lens, q_pos_offsets, num_rows, total_query,
                             nullptr, nullptr, total_query, nullptr, num_q_heads, num_kv_heads, head_dim, dtype,
                             scale, is_causal, 0, out, out_stride_token, out_stride_head, lse, lse_stride_token,
                             workspace, workspace_bytes, err, stream);
  }
  const int pair_queries = 2 * (128 / group);
  const int64_t cap = unit_bound(num_rows, total_query, num_kv_heads, pair_queries);
  SEB_CHECK_ARG(cap < (1ll << 30), "seb_paged_attention: batch too large");
  const RouteLayout l = route_layout(num_rows, cap);
  char* ws = static_cast<char*>(workspace);
  RouteParams r;
  r.q_lens = q_lens;
  r.k_lens = k_lens;
  r.q_starts = q_starts;
  r.num_rows = num_rows;
  r.max_blocks = max_blocks;
  r.hkv = num_kv_heads;
  r.pair_queries = pair_queries;
  r.unit_cap = (int32_t)cap;
  r.counts = reinterpret_cast<int32_t*>(ws + l.counts);
  r.dec_tokens = reinterpret_cast<int32_t*>(ws + l.dec_tokens);
  r.dec_rows = reinterpret_cast<int32_t*>(ws + l.dec_rows);
  r.units = reinterpret_cast<int32_t*>(ws + l.units);
  r.err = err;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  route_rows_kernel<<<1, kRouteThreads, 0, s>>>(r);
  int rc = launch_status("route_rows_kernel");
  if (rc != SEB_OK) return rc;
  rc = paged_decode_impl(q, q_stride_token, q_stride_head, k_cache, v_cache, num_blocks, block_table,
                         block_table_stride, max_blocks, q_starts, k_lens, q_pos_offsets, num_rows, total_query,
                         r.dec_tokens, r.dec_rows, num_rows, r.counts, num_q_heads, num_kv_heads, head_dim, dtype,
                         scale, is_causal, 0, out, out_stride_token, out_stride_head, lse, lse_stride_token,
                         ws + l.bytes, workspace_bytes - l.bytes, err, stream);
  if (rc != SEB_OK) return rc;
  return paged_prefill_impl(q, q_stride_token, q_stride_head, k_cache, v_cache, num_blocks, block_table,
                            block_table_stride, max_blocks, q_starts, q_lens, k_lens, q_pos_offsets, num_rows,
                            total_query, nullptr, 0, 0, num_q_heads, num_kv_heads, head_dim, dtype, scale, is_causal,
                            out, out_stride_token, out_stride_head, lse, lse_stride_token, err, stream, r.units,
                            r.counts + 1, (int32_t)cap);
}
