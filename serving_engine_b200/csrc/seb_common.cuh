// Shared helpers for the sm_100a kernels of serving_engine_b200: element traits,
// host-side status/error plumbing and the inline-PTX primitives the kernels use
// (mbarrier, 1-D bulk async copy, proxy fences, ldmatrix/movmatrix, mma.sync).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/serving_engine_b200.h"

namespace seb {

constexpr int kBlockSize = SEB_BLOCK_SIZE;

// ---------------------------------------------------------------- host errors
// One message buffer per host thread; seb_last_error() returns it.
void set_error(const char* fmt, ...);
void clear_error();

#define SEB_CHECK_ARG(cond, ...)     \
  do {                               \
    if (!(cond)) {                   \
      ::seb::set_error(__VA_ARGS__); \
      return SEB_EINVAL;             \
    }                                \
  } while (0)

#define SEB_CHECK_CUDA(expr)                                                    \
  do {                                                                          \
    cudaError_t _e = (expr);                                                    \
    if (_e != cudaSuccess) {                                                    \
      ::seb::set_error("%s failed: %s", #expr, cudaGetErrorString(_e));         \
      return SEB_ECUDA;                                                         \
    }                                                                           \
  } while (0)

inline int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s launch failed: %s", what, cudaGetErrorString(e));
    return SEB_ECUDA;
  }
  return SEB_OK;
}

inline int elem_size(int dtype) {
  switch (dtype) {
    case SEB_F32: return 4;
    case SEB_F16: return 2;
    case SEB_BF16: return 2;
    default: return 0;
  }
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Number of SMs of the current device (cached per device id).
int num_sms();

// Raises Kernel's dynamic shared-memory limit to `bytes` once per device (the
// attribute is per device context). Safe when several host threads launch at
// once: the first caller per device sets it under a lock, later callers see the
// published flag.
template <auto Kernel>
int set_smem_limit_once(int bytes) {
  constexpr int kMaxDevices = 64;
  static std::atomic<bool> done[kMaxDevices];
  static std::mutex mu;
  int dev = 0;
  SEB_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) {
    SEB_CHECK_CUDA(cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    return SEB_OK;
  }
  if (done[dev].load(std::memory_order_acquire)) return SEB_OK;
  std::lock_guard<std::mutex> lk(mu);
  if (!done[dev].load(std::memory_order_relaxed)) {
    SEB_CHECK_CUDA(cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done[dev].store(true, std::memory_order_release);
  }
  return SEB_OK;
}

// ------------------------------------------------------------- element traits
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_float(float x) { return x; }
  static __device__ __forceinline__ float from_float(float x) { return x; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_float(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_float(float x) { return __float2bfloat16_rn(x); }
};

// --------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes mbarrier.init visible to the async proxy (bulk copies complete_tx on it).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with acquire at cluster scope, for barriers that receive arrivals
// (with release at cluster scope) from the other CTAs of a cluster.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_bounded_cluster(uint32_t bar, uint32_t parity,
                                                          uint32_t limit = (1u << 18)) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
  }
  return false;
}

// Non-blocking check of a phase.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait whose suspension lasts at most about `hint_ns` nanoseconds.
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `limit` polls and returns false so the caller can
// report SEB_ERRBIT_TIMEOUT instead of hanging the GPU. Each unsatisfied try_wait
// suspends the thread for a hardware-defined slice, measured at about 4 us on
// B200, so the default bound is about one second; waits that are satisfied
// return at once.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  uint32_t limit = (1u << 18)) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  return false;
}

// ---- thread-block clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of shared offset `addr` in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Arrive on an mbarrier given by its shared::cluster address (which may be in
// another CTA of the cluster), with the default semantics of mbarrier.arrive.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// Whole-cluster barrier (every thread of every CTA arrives, then waits).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Orders this thread's prior generic-proxy shared-memory accesses before
// subsequent async-proxy (bulk copy / tensor core) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1-D bulk copy global -> shared, completion counted in bytes on `bar`.
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Transpose an 8x8 b16 matrix held in the standard fragment layout
// (thread g*4+t holds row g, columns 2t and 2t+1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

template <typename T> struct Mma;

template <> struct Mma<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t v) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&v));
  }
};

template <> struct Mma<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t v) {
    return __half22float2(*reinterpret_cast<__half2*>(&v));
  }
};

__device__ __forceinline__ void atomic_or_err(int32_t* err, uint32_t bit) {
  if (err) atomicOr(err, static_cast<int32_t>(bit));
}

__device__ __forceinline__ float warp_max_xor(float v, int lanemask_lo, int lanemask_hi) {
  for (int o = lanemask_lo; o <= lanemask_hi; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum_xor(float v, int lanemask_lo, int lanemask_hi) {
  for (int o = lanemask_lo; o <= lanemask_hi; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------- launchers shared across files
// seb_paged_decode with an optional device-side item count: items at or past
// *num_items_dev (num_items bounds it and sizes the grid) exit at once.
int paged_decode_impl(const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* k_cache,
                      const void* v_cache, int64_t num_blocks, const int32_t* block_table, int64_t block_table_stride,
                      int64_t max_blocks, const int32_t* q_starts, const int32_t* k_lens, const int32_t* q_pos_offsets,
                      int32_t num_rows, int32_t total_query, const int32_t* item_query, const int32_t* item_row,
                      int32_t num_items, const int32_t* num_items_dev, int32_t num_q_heads, int32_t num_kv_heads,
                      int32_t head_dim, int32_t dtype, float scale, int32_t is_causal, int32_t blocks_per_split,
                      void* out, int64_t out_stride_token, int64_t out_stride_head, float* lse,
                      int64_t lse_stride_token, void* workspace, int64_t workspace_bytes, int32_t* err,
                      void* stream);

// seb_paged_prefill with an optional device-built unit list: unit u < *num_units
// (<= unit_cap, which sizes the grid) is row unit_list[2u], kv head
// unit_list[2u+1] & 255 and Q-tile pair unit_list[2u+1] >> 8.
int paged_prefill_impl(const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* k_cache,
                       const void* v_cache, int64_t num_blocks, const int32_t* block_table,
                       int64_t block_table_stride, int64_t max_blocks, const int32_t* q_starts,
                       const int32_t* q_lens, const int32_t* k_lens, const int32_t* q_pos_offsets, int32_t num_rows,
                       int32_t total_query, const int32_t* rows, int32_t num_prefill_rows, int32_t max_q_len,
                       int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t dtype, float scale,
                       int32_t is_causal, void* out, int64_t out_stride_token, int64_t out_stride_head, float* lse,
                       int64_t lse_stride_token, int32_t* err, void* stream, const int32_t* unit_list,
                       const int32_t* num_units, int32_t unit_cap);

}  // namespace seb
