// 16-byte element vectors and the row-sum step of RMSNorm, shared by the
// residual add + RMSNorm kernel and the all-reduce fused with it, so that both
// round and reduce in exactly the same order (their outputs are bit-identical
// for the same summed row).
#pragma once

#include "seb_common.cuh"

namespace seb {

// 8 elements of a 16-bit type in one 16-byte word.
template <typename T>
struct Vec8 {
  uint4 raw;
  __device__ __forceinline__ float get(int i) const {
    return Elem<T>::to_float(reinterpret_cast<const T*>(&raw)[i]);
  }
  __device__ __forceinline__ void set(int i, float v) { reinterpret_cast<T*>(&raw)[i] = Elem<T>::from_float(v); }
};

// Sum of `v` over the THREADS threads of the block: a butterfly inside each
// warp, then the warps' sums added in warp order. `red` holds THREADS / 32
// floats; the caller syncs the block before `red` is written again.
template <int THREADS>
__device__ __forceinline__ float block_sum_ordered(float v, float* red) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < THREADS / 32; ++k) tot += red[k];
  return tot;
}

// RMSNorm of one row held as kMaxVec 16-byte vectors per thread (vector i of
// the row at thread i % THREADS, slot i / THREADS): returns the fp32 scale
// rsqrt(mean(x^2) + eps), with x^2 accumulated per thread in slot order.
template <typename T, int THREADS, int kMaxVec>
__device__ __forceinline__ float rms_scale(const Vec8<T> (&v)[kMaxVec], int nvec, int hidden, float eps,
                                           float* red) {
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    if ((int)threadIdx.x + k * THREADS < nvec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[k].get(e), v[k].get(e), ss);
    }
  }
  return rsqrtf(block_sum_ordered<THREADS>(ss, red) / (float)hidden + eps);
}

}  // namespace seb
