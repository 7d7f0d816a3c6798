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
  uint64_t dims[3], strides[2];
  uint32_t box[3];
  int dtype, device;
  CUtensorMap map;
  bool used;
};

constexpr int kCacheSize = 32;
Entry g_cache[kCacheSize];
int g_next = 0;
std::mutex g_mu;

bool same(const Entry& e, const void* base, int dtype, int dev, const uint64_t dims[3], const uint64_t strides[2],
          const uint32_t box[3]) {
  return e.used && e.base == base && e.dtype == dtype && e.device == dev && e.dims[0] == dims[0] &&
         e.dims[1] == dims[1] && e.dims[2] == dims[2] && e.strides[0] == strides[0] && e.strides[1] == strides[1] &&
         e.box[0] == box[0] && e.box[1] == box[1] && e.box[2] == box[2];
}

}  // namespace

int tensor_map_3d(CUtensorMap* out, const void* base, int dtype, const uint64_t dims[3], const uint64_t strides[2],
                  const uint32_t box[3]) {
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto& e : g_cache) {
      if (same(e, base, dtype, dev, dims, strides, box)) {
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
    set_error("tensor_map_3d: 16-bit dtype required");
    return SEB_EINVAL;
  }
  const CUtensorMapDataType ty = dtype == SEB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t gdims[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t gstrides[2] = {strides[0], strides[1]};
  cuuint32_t gbox[3] = {box[0], box[1], box[2]};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap map;
  CUresult r = fn(&map, ty, 3, const_cast<void*>(base), gdims, gstrides, gbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (CUresult %d) for %p dims (%llu, %llu, %llu) strides (%llu, %llu)",
              (int)r, base, (unsigned long long)dims[0], (unsigned long long)dims[1], (unsigned long long)dims[2],
              (unsigned long long)strides[0], (unsigned long long)strides[1]);
    return SEB_ECUDA;
  }
  std::memcpy(out, &map, sizeof(CUtensorMap));
  std::lock_guard<std::mutex> lk(g_mu);
  Entry& e = g_cache[g_next];
  g_next = (g_next + 1) % kCacheSize;
  e.base = base;
  for (int i = 0; i < 3; ++i) {
    e.dims[i] = dims[i];
    e.box[i] = box[i];
  }
  e.strides[0] = strides[0];
  e.strides[1] = strides[1];
  e.dtype = dtype;
  e.device = dev;
  std::memcpy(&e.map, &map, sizeof(CUtensorMap));
  e.used = true;
  return SEB_OK;
}

int kv_tensor_map(CUtensorMap* out, const void* base, int dtype, int64_t num_blocks, int num_kv_heads,
                  int head_dim) {
  if (head_dim % 64 != 0) {
    set_error("kv_tensor_map: head_dim must be a multiple of 64");
    return SEB_EUNSUPPORTED;
  }
  const uint64_t dims[3] = {(uint64_t)head_dim, (uint64_t)num_kv_heads, (uint64_t)num_blocks * kBlockSize};
  const uint64_t strides[2] = {(uint64_t)head_dim * 2, (uint64_t)head_dim * 2 * num_kv_heads};
  const uint32_t box[3] = {64, 1, (uint32_t)kBlockSize};
  return tensor_map_3d(out, base, dtype, dims, strides, box);
}

}  // namespace seb
