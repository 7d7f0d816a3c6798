// Host-side creation and caching of the KV-pool tensor maps.
#include "seb_tma.cuh"

#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

namespace seb {
namespace {

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

struct Entry {
  const void* base;
  int64_t num_blocks;
  int hkv, d, dtype, device;
  CUtensorMap map;
  bool used;
};

constexpr int kCacheSize = 16;
Entry g_cache[kCacheSize];
int g_next = 0;
std::mutex g_mu;

}  // namespace

int kv_tensor_map(CUtensorMap* out, const void* base, int dtype, int64_t num_blocks, int num_kv_heads,
                  int head_dim) {
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto& e : g_cache) {
      if (e.used && e.base == base && e.num_blocks == num_blocks && e.hkv == num_kv_heads && e.d == head_dim &&
          e.dtype == dtype && e.device == dev) {
        std::memcpy(out, &e.map, sizeof(CUtensorMap));
        return SEB_OK;
      }
    }
  }
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled unavailable from the CUDA driver");
    return SEB_ECUDA;
  }
  if (dtype != SEB_BF16 && dtype != SEB_F16) {
    set_error("kv_tensor_map: 16-bit dtype required");
    return SEB_EINVAL;
  }
  if (head_dim % 64 != 0) {
    set_error("kv_tensor_map: head_dim must be a multiple of 64");
    return SEB_EUNSUPPORTED;
  }
  const CUtensorMapDataType ty = dtype == SEB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {(cuuint64_t)head_dim, (cuuint64_t)num_kv_heads, (cuuint64_t)num_blocks * kBlockSize};
  cuuint64_t strides[2] = {(cuuint64_t)head_dim * 2, (cuuint64_t)head_dim * 2 * num_kv_heads};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)kBlockSize};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap map;
  CUresult r = fn(&map, ty, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (CUresult %d) for pool %p, %lld blocks, %d heads, dim %d", (int)r, base,
              (long long)num_blocks, num_kv_heads, head_dim);
    return SEB_ECUDA;
  }
  std::memcpy(out, &map, sizeof(CUtensorMap));
  std::lock_guard<std::mutex> lk(g_mu);
  Entry& e = g_cache[g_next];
  g_next = (g_next + 1) % kCacheSize;
  e.base = base;
  e.num_blocks = num_blocks;
  e.hkv = num_kv_heads;
  e.d = head_dim;
  e.dtype = dtype;
  e.device = dev;
  std::memcpy(&e.map, &map, sizeof(CUtensorMap));
  e.used = true;
  return SEB_OK;
}

}  // namespace seb
