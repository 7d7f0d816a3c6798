// Fused KV append: scatters the new K and V rows of one layer into their
// slot_mapping positions of the paged pool in ONE launch.
//
// Replaces _PagedKVCache.write (serving_engine/model_runner.py:21-32): two
// index_copy_ launches over the flat [num_blocks*16, num_kv_heads, head_dim]
// views, plus the transpose copies HF's [1, kv_heads, seq, dim] layout forces.
// Here the source is read through its strides, so no staging copy is made.
//
// Roofline: HBM, 2 * n_tokens * num_kv_heads * head_dim * elem bytes read and
// the same written. Decode-sized calls (tens of tokens) are launch-latency bound.
// One warp copies one token's K (or V) rows of every kv head.
#include "seb_common.cuh"

namespace seb {
namespace {

template <int VEC> struct VecType;
template <> struct VecType<16> { using T = uint4; };
template <> struct VecType<8> { using T = uint2; };
template <> struct VecType<4> { using T = uint32_t; };
template <> struct VecType<2> { using T = uint16_t; };

struct AppendParams {
  const char* src[2];        // K, V base pointers
  int64_t st_tok[2];         // bytes
  int64_t st_head[2];        // bytes
  char* dst[2];              // k_cache, v_cache
  const int64_t* slots;
  int64_t n_tokens;
  int64_t num_slots;
  int64_t row_bytes;         // head_dim * elem
  int32_t num_kv_heads;
  int32_t cph_shift;  // log2(row_bytes / VEC) when a power of two, else -1
  int32_t* err;
};

// One warp per (token t, plane kv): the token's num_kv_heads rows land
// contiguously in its slot, so the warp's stores cover one contiguous range;
// loads follow the source's token/head strides. Chunk c of the slot is head
// c / chunks_per_head, offset c % chunks_per_head.
template <int VEC>
__global__ void __launch_bounds__(256) kv_append_kernel(AppendParams p) {
  using V = typename VecType<VEC>::T;
  const int64_t wid = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t t = wid >> 1;
  const int kv = (int)(wid & 1);
  if (t >= p.n_tokens) return;
  const int64_t slot = __ldg(p.slots + t);
  if (slot < 0 || slot >= p.num_slots) {
    if (lane == 0 && kv == 0) atomic_or_err(p.err, SEB_ERRBIT_SLOT);
    return;
  }
  const int cph = (int)(p.row_bytes / VEC);  // chunks per head row
  const int chunks = p.num_kv_heads * cph;
  const char* src = p.src[kv] + t * p.st_tok[kv];
  V* dst = reinterpret_cast<V*>(p.dst[kv] + slot * p.num_kv_heads * p.row_bytes);
  const int64_t sth = p.st_head[kv];
  constexpr int U = 4;
  for (int c0 = lane; c0 < chunks; c0 += 32 * U) {
    V v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + 32 * u;
      if (c < chunks) {
        const int h = p.cph_shift >= 0 ? (c >> p.cph_shift) : c / cph;
        v[u] = __ldg(reinterpret_cast<const V*>(src + h * sth) + (c - h * cph));
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + 32 * u;
      if (c < chunks) dst[c] = v[u];
    }
  }
}

}  // namespace
}  // namespace seb

extern "C" int seb_kv_append(const void* k_new, int64_t k_stride_token, int64_t k_stride_head,
                             const void* v_new, int64_t v_stride_token, int64_t v_stride_head,
                             int64_t n_tokens, const int64_t* slot_mapping, void* k_cache,
                             void* v_cache, int64_t num_blocks, int32_t num_kv_heads,
                             int32_t head_dim, int32_t dtype, int32_t* err, void* stream) {
  using namespace seb;
  clear_error();
  const int es = elem_size(dtype);
  SEB_CHECK_ARG(es > 0, "seb_kv_append: unknown dtype %d", dtype);
  SEB_CHECK_ARG(n_tokens >= 0, "seb_kv_append: n_tokens < 0");
  SEB_CHECK_ARG(num_blocks > 0 && num_kv_heads > 0 && head_dim > 0,
                "seb_kv_append: num_blocks, num_kv_heads, head_dim must be positive");
  if (n_tokens == 0) return SEB_OK;
  SEB_CHECK_ARG(k_new && v_new && slot_mapping && k_cache && v_cache,
                "seb_kv_append: NULL pointer argument");

  AppendParams p;
  p.src[0] = static_cast<const char*>(k_new);
  p.src[1] = static_cast<const char*>(v_new);
  p.st_tok[0] = k_stride_token * es;
  p.st_tok[1] = v_stride_token * es;
  p.st_head[0] = k_stride_head * es;
  p.st_head[1] = v_stride_head * es;
  p.dst[0] = static_cast<char*>(k_cache);
  p.dst[1] = static_cast<char*>(v_cache);
  p.slots = slot_mapping;
  p.n_tokens = n_tokens;
  p.num_slots = num_blocks * kBlockSize;
  p.row_bytes = (int64_t)head_dim * es;
  p.num_kv_heads = num_kv_heads;
  p.err = err;

  // Widest vector every address and stride allows.
  int vec = 16;
  auto ok = [&](int v) {
    for (int i = 0; i < 2; ++i) {
      if (!aligned(p.src[i], v) || !aligned(p.dst[i], v)) return false;
      if (p.st_tok[i] % v || p.st_head[i] % v) return false;
    }
    return p.row_bytes % v == 0;
  };
  while (vec > es && !ok(vec)) vec >>= 1;
  SEB_CHECK_ARG(ok(vec), "seb_kv_append: pointers or strides not aligned to the element size");

  const int64_t cph = p.row_bytes / vec;
  p.cph_shift = -1;
  for (int sh = 0; sh < 31; ++sh)
    if ((1ll << sh) == cph) p.cph_shift = sh;
  SEB_CHECK_ARG((int64_t)num_kv_heads * cph < (1ll << 30), "seb_kv_append: row too large");
  const int64_t warps = n_tokens * 2;
  const int64_t blocks = (warps + 7) / 8;
  SEB_CHECK_ARG(blocks < (1ll << 31), "seb_kv_append: too many tokens");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (vec) {
    case 16: kv_append_kernel<16><<<(unsigned)blocks, 256, 0, s>>>(p); break;
    case 8: kv_append_kernel<8><<<(unsigned)blocks, 256, 0, s>>>(p); break;
    case 4: kv_append_kernel<4><<<(unsigned)blocks, 256, 0, s>>>(p); break;
    default: kv_append_kernel<2><<<(unsigned)blocks, 256, 0, s>>>(p); break;
  }
  return launch_status("kv_append_kernel");
}
