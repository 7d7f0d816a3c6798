// Batched copy-on-write block copy across every layer and both K/V planes of
// the engine's pool kv_cache[L, 2, num_blocks, 16, H, D] (model_runner.py:101-110).
//
// New relative to the reference: BlockManager.fork (block_manager.py:129-132)
// only shares tables and bumps refcounts. A prefix-cache fork whose last shared
// block is partially filled must copy that block before the child appends into
// it; this op performs all such copies of a step in one launch.
//
// Roofline: HBM, n_pairs * L * 2 * block_bytes read and the same written.
#include "seb_common.cuh"

namespace seb {
namespace {

template <int VEC> struct CopyVec;
template <> struct CopyVec<16> { using T = uint4; };
template <> struct CopyVec<8> { using T = uint2; };
template <> struct CopyVec<4> { using T = uint32_t; };
template <> struct CopyVec<2> { using T = uint16_t; };

struct CopyParams {
  char* pool;
  int64_t num_layers;
  int64_t layer_stride;  // bytes between layer l and l+1
  int64_t plane_stride;  // bytes between K and V planes of one layer = num_blocks * block_bytes
  int64_t num_blocks;
  int64_t block_bytes;
  const int64_t* src;
  const int64_t* dst;
  int64_t n_pairs;
  int32_t* err;
};

// Thread u copies chunk c of (pair i, layer l, plane p), u = ((i*L + l)*2 + p)*chunks + c.
template <int VEC>
__global__ void __launch_bounds__(256) copy_blocks_kernel(CopyParams p) {
  using V = typename CopyVec<VEC>::T;
  const int64_t chunks = p.block_bytes / VEC;
  const int64_t per_pair = p.num_layers * 2 * chunks;
  const int64_t total = p.n_pairs * per_pair;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = u / per_pair;
    int64_t r = u - i * per_pair;
    const int64_t lp = r / chunks;
    const int64_t c = r - lp * chunks;
    const int64_t l = lp >> 1;
    const int64_t pl = lp & 1;
    const int64_t s = __ldg(p.src + i);
    const int64_t d = __ldg(p.dst + i);
    if (s < 0 || s >= p.num_blocks || d < 0 || d >= p.num_blocks) {
      if (lp == 0 && c == 0) atomic_or_err(p.err, SEB_ERRBIT_BLOCK_ID);
      continue;
    }
    char* base = p.pool + l * p.layer_stride + pl * p.plane_stride;
    const V* sp = reinterpret_cast<const V*>(base + s * p.block_bytes) + c;
    V* dp = reinterpret_cast<V*>(base + d * p.block_bytes) + c;
    *dp = *sp;
  }
}

}  // namespace
}  // namespace seb

extern "C" int seb_copy_blocks(void* kv_cache, int64_t num_layers, int64_t layer_stride_bytes,
                               int64_t num_blocks, int64_t block_bytes, const int64_t* src,
                               const int64_t* dst, int64_t n_pairs, int32_t* err, void* stream) {
  using namespace seb;
  clear_error();
  SEB_CHECK_ARG(n_pairs >= 0 && num_layers >= 0, "seb_copy_blocks: negative count");
  if (n_pairs == 0 || num_layers == 0) return SEB_OK;
  SEB_CHECK_ARG(kv_cache && src && dst, "seb_copy_blocks: NULL pointer argument");
  SEB_CHECK_ARG(num_blocks > 0 && block_bytes > 0, "seb_copy_blocks: empty pool");
  CopyParams p;
  p.pool = static_cast<char*>(kv_cache);
  p.num_layers = num_layers;
  p.layer_stride = layer_stride_bytes;
  p.plane_stride = num_blocks * block_bytes;
  p.num_blocks = num_blocks;
  p.block_bytes = block_bytes;
  p.src = src;
  p.dst = dst;
  p.n_pairs = n_pairs;
  p.err = err;
  int vec = 16;
  while (vec > 2 && (!aligned(kv_cache, vec) || block_bytes % vec || layer_stride_bytes % vec))
    vec >>= 1;
  SEB_CHECK_ARG(aligned(kv_cache, vec) && block_bytes % vec == 0 && layer_stride_bytes % vec == 0,
                "seb_copy_blocks: pool not 2-byte aligned");
  const int64_t total = n_pairs * num_layers * 2 * (block_bytes / vec);
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (vec) {
    case 16: copy_blocks_kernel<16><<<(unsigned)blocks, 256, 0, s>>>(p); break;
    case 8: copy_blocks_kernel<8><<<(unsigned)blocks, 256, 0, s>>>(p); break;
    case 4: copy_blocks_kernel<4><<<(unsigned)blocks, 256, 0, s>>>(p); break;
    default: copy_blocks_kernel<2><<<(unsigned)blocks, 256, 0, s>>>(p); break;
  }
  return launch_status("copy_blocks_kernel");
}
