// TMA (tensor memory accelerator) helpers: host-side tensor-map creation for the
// paged KV pool and the device-side tiled bulk-tensor load.
#pragma once

#include <cuda.h>

#include "seb_common.cuh"

namespace seb {

// Tensor map over one layer's K (or V) pool [num_blocks * 16 rows, num_kv_heads, head_dim]
// of 16-bit elements, viewed as 3-D (head_dim, num_kv_heads, rows) with a box of
// (64 elements, 1 head, 16 rows) and 128-byte swizzling: one load brings a 2 KB
// 16 x 128-byte panel of one block and one kv head into shared memory, laid out
// as the 128B-swizzled rows ldmatrix reads without bank conflicts.
// Returns SEB_OK or an SEB_E* status (with seb_last_error set). Results are
// cached per (pointer, shape), so repeated calls on the same pool cost a lookup.
int kv_tensor_map(CUtensorMap* out, const void* base, int dtype, int64_t num_blocks, int num_kv_heads,
                  int head_dim);

// General 3-D map of 16-bit elements with 128-byte swizzling: dims (innermost
// first) in elements, strides of dims 1 and 2 in bytes, box in elements
// (box[0] * 2 <= 128). Cached like kv_tensor_map.
int tensor_map_3d(CUtensorMap* out, const void* base, int dtype, const uint64_t dims[3],
                  const uint64_t strides[2], const uint32_t box[3]);

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

// The CTA-pair form: the copy lands in this CTA's shared memory at `dst` and
// completes its bytes on the mbarrier `bar_cluster` (a shared::cluster address,
// which may belong to the pair's other CTA).
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar_cluster)
      : "memory");
}

// Tiled store of a box from this CTA's shared memory (laid out as the map's
// swizzle expects) to global memory, tracked by the issuing thread's bulk
// groups. Coordinates must be non-negative; boxes past the tensor's end clip.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The issuing thread's committed stores have read their shared-memory source.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// The issuing thread's committed stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

}  // namespace seb
