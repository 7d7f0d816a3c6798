// All-reduce(SUM) fused with the residual add and RMSNorm that follow it in the
// tensor-parallel decoder (after o_proj and after down_proj), over CUDA IPC peer
// memory: plain loads and stores across NVLink, no multicast, no library call.
//
// Two-shot schedule. Rank r owns token rows [r*T/N, (r+1)*T/N). For each of its
// rows it
//   1. reads the row of every rank's partial sum (its own from local HBM, the
//      others over NVLink) and adds them in fp32 in rank order, rounding the sum
//      once to the element type: the value an all-reduce of the 16-bit tensor
//      returns;
//   2. adds that to its residual row (rounded, like the eager add) and
//      normalises the result exactly as seb_add_rmsnorm does;
//   3. stores the new residual row and the normalised row into every rank's
//      buffers.
// Every rank therefore ends with bit-identical residual and normalised tensors.
// Per rank and call that is (N-1)/N of one partial read over NVLink and 2(N-1)/N
// of one tensor written over it, against 2(N-1)/N read and written by a ring
// all-reduce followed by a separate add + norm pass.
//
// Ordering, per rank's flag words (in its peer memory):
//   ready[src] = e: rank src has entered call e, so its partial for call e is
//                written (by the kernels before this one on its stream) and its
//                call e-1, with every read of its residual / output buffers
//                after it, is over; peers may read its partial and write its rows.
//   done[src]  = e: every row of rank src has been stored on every rank.
// A call's last CTA on a rank publishes done, waits for every peer's done, and
// advances the rank's epoch, so no rank rewrites its partial (next GEMM) while a
// peer still reads it, and the kernels after this one see every pushed row. The
// epoch lives in device memory, so a CUDA graph replays the calls unchanged.
// Every wait is bounded: when it gives up the kernel sets SEB_ERRBIT_TIMEOUT
// and goes on without the data (the result is then invalid, and the host
// raises), so a rank that never arrives cannot hang the GPU.
#include "seb_common.cuh"
#include "seb_vec.cuh"

#include <algorithm>
#include <cstring>

namespace seb {
namespace {

constexpr int kReady = 0;            // flag words [0, 64): ready[src]
constexpr int kDone = 64;            // [64, 128): done[src]
constexpr int kEpoch = 128;          // this rank's completed calls
constexpr int kArrival = 129;        // CTAs of the running call that are finished
constexpr uint32_t kDefaultPolls = 1u << 22;  // about 1-4 s: each poll sleeps ~0.25 us plus a load

static_assert(SEB_PEER_FLAG_BYTES >= (kArrival + 1) * 4, "flag region too small");
static_assert(SEB_MAX_PEERS <= 64, "ready/done hold 64 ranks");

struct PeerNormParams {
  const void* partial[SEB_MAX_PEERS];
  void* x[SEB_MAX_PEERS];
  void* out[SEB_MAX_PEERS];
  uint32_t* flags[SEB_MAX_PEERS];
  const void* w;
  int64_t tokens;
  int hidden;
  float eps;
  int rank;  // rank of blockIdx.y == 0; blockIdx.y > 0 only in the all-ranks (one device) launch
  int world;
  uint32_t polls;
  int32_t* err;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Waits until *f has reached `target` (wrap-safe), at most `polls` polls.
__device__ __forceinline__ bool wait_reached(const uint32_t* f, uint32_t target, uint32_t polls) {
  for (uint32_t i = 0; i < polls; ++i) {
    if ((int32_t)(ld_acquire_sys(f) - target) >= 0) return true;
    __nanosleep(256);
  }
  return false;
}

template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS) allreduce_add_rmsnorm_kernel(PeerNormParams p) {
  constexpr int kMaxVec = 4;
  __shared__ float red[THREADS / 32];
  __shared__ uint32_t s_epoch;
  const int rank = p.rank + (int)blockIdx.y;
  const int world = p.world;
  uint32_t* my = p.flags[rank];
  const int tid = threadIdx.x;
  if (tid == 0) s_epoch = *reinterpret_cast<volatile uint32_t*>(my + kEpoch) + 1u;
  __syncthreads();
  const uint32_t e = s_epoch;

  // 1. announce this rank's partial, wait for the peers'
  if (blockIdx.x == 0 && tid < world && tid != rank) st_release_sys(p.flags[tid] + kReady + rank, e);
  if (tid < world && tid != rank && !wait_reached(my + kReady + tid, e, p.polls))
    atomic_or_err(p.err, SEB_ERRBIT_TIMEOUT);
  __syncthreads();

  // 2. this rank's rows: sum, add, normalise, store everywhere
  const int64_t r0 = p.tokens * rank / world, r1 = p.tokens * (rank + 1) / world;
  const int nvec = p.hidden / 8;
  const uint4* wv = static_cast<const uint4*>(p.w);
  const uint4* xr_all = static_cast<const uint4*>(p.x[rank]);
  for (int64_t row = r0 + blockIdx.x; row < r1; row += gridDim.x) {
    const int64_t base = row * nvec;
    Vec8<T> v[kMaxVec];
#pragma unroll
    for (int k = 0; k < kMaxVec; ++k) {
      const int i = tid + k * THREADS;
      if (i < nvec) {
        uint4 part[SEB_MAX_PEERS];
#pragma unroll
        for (int q = 0; q < SEB_MAX_PEERS; ++q)
          if (q < world) part[q] = __ldcg(static_cast<const uint4*>(p.partial[q]) + base + i);
        float s[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j] = 0.f;
#pragma unroll
        for (int q = 0; q < SEB_MAX_PEERS; ++q) {
          if (q < world) {
            Vec8<T> pq;
            pq.raw = part[q];
#pragma unroll
            for (int j = 0; j < 8; ++j) s[j] += pq.get(j);
          }
        }
        Vec8<T> sum;
#pragma unroll
        for (int j = 0; j < 8; ++j) sum.set(j, s[j]);  // the all-reduce result, rounded once
        v[k].raw = xr_all[base + i];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[k].set(j, v[k].get(j) + sum.get(j));  // rounded, like the eager add
      }
    }
    const float r = rms_scale<T, THREADS, kMaxVec>(v, nvec, p.hidden, p.eps, red);
#pragma unroll
    for (int k = 0; k < kMaxVec; ++k) {
      const int i = tid + k * THREADS;
      if (i < nvec) {
        Vec8<T> wk, o;
        wk.raw = __ldg(wv + i);
#pragma unroll
        for (int j = 0; j < 8; ++j) o.set(j, v[k].get(j) * r * wk.get(j));
#pragma unroll
        for (int q = 0; q < SEB_MAX_PEERS; ++q) {
          if (q < world) {
            static_cast<uint4*>(p.x[q])[base + i] = v[k].raw;
            static_cast<uint4*>(p.out[q])[base + i] = o.raw;
          }
        }
      }
    }
    __syncthreads();  // `red` is rewritten by the next row
  }

  // 3. the last CTA of this rank publishes done, waits for the peers', closes the call
  if (tid == 0) {
    __threadfence_system();
    const uint32_t prev = atomicAdd(my + kArrival, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int q = 0; q < world; ++q)
        if (q != rank) st_release_sys(p.flags[q] + kDone + rank, e);
      for (int q = 0; q < world; ++q)
        if (q != rank && !wait_reached(my + kDone + q, e, p.polls)) atomic_or_err(p.err, SEB_ERRBIT_TIMEOUT);
      *reinterpret_cast<volatile uint32_t*>(my + kArrival) = 0u;
      *reinterpret_cast<volatile uint32_t*>(my + kEpoch) = e;
    }
  }
}

template <typename T, int THREADS>
int launch_peer_norm(const PeerNormParams& p, bool all_ranks, cudaStream_t s) {
  const int64_t rows = (p.tokens + p.world - 1) / p.world;  // most rows a rank owns
  const int gx = (int)std::max<int64_t>(1, std::min<int64_t>(rows, 4 * (int64_t)num_sms()));
  if (!all_ranks) {
    allreduce_add_rmsnorm_kernel<T, THREADS><<<gx, THREADS, 0, s>>>(p);
    return launch_status("allreduce_add_rmsnorm_kernel");
  }
  // every rank's CTAs in one launch on this device; they wait on one another,
  // so the launch is cooperative (all CTAs resident, or the launch is refused)
  PeerNormParams q = p;
  void* args[] = {&q};
  SEB_CHECK_CUDA(cudaLaunchCooperativeKernel((const void*)allreduce_add_rmsnorm_kernel<T, THREADS>,
                                             dim3(gx, p.world), dim3(THREADS), args, 0, s));
  return SEB_OK;
}

}  // namespace
}  // namespace seb

extern "C" int seb_peer_alloc(size_t bytes, void** ptr) {
  using namespace seb;
  clear_error();
  SEB_CHECK_ARG(ptr != nullptr && bytes > 0, "seb_peer_alloc: bad arguments");
  void* p = nullptr;
  SEB_CHECK_CUDA(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    set_error("seb_peer_alloc: cudaMemset failed: %s", cudaGetErrorString(e));
    return SEB_ECUDA;
  }
  *ptr = p;
  return SEB_OK;
}

extern "C" int seb_peer_free(void* ptr) {
  using namespace seb;
  clear_error();
  SEB_CHECK_CUDA(cudaFree(ptr));
  return SEB_OK;
}

extern "C" int seb_peer_export(void* ptr, void* handle) {
  using namespace seb;
  clear_error();
  static_assert(sizeof(cudaIpcMemHandle_t) == SEB_PEER_HANDLE_BYTES, "IPC handle size");
  SEB_CHECK_ARG(ptr != nullptr && handle != nullptr, "seb_peer_export: NULL argument");
  cudaIpcMemHandle_t h;
  SEB_CHECK_CUDA(cudaIpcGetMemHandle(&h, ptr));
  memcpy(handle, &h, sizeof(h));
  return SEB_OK;
}

extern "C" int seb_peer_import(const void* handle, void** ptr) {
  using namespace seb;
  clear_error();
  SEB_CHECK_ARG(ptr != nullptr && handle != nullptr, "seb_peer_import: NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  SEB_CHECK_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return SEB_OK;
}

extern "C" int seb_peer_close(void* ptr) {
  using namespace seb;
  clear_error();
  SEB_CHECK_CUDA(cudaIpcCloseMemHandle(ptr));
  return SEB_OK;
}

extern "C" int seb_allreduce_add_rmsnorm(void* const* partial, void* const* x, void* const* out,
                                         void* const* flags, const void* weight, int64_t n_tokens,
                                         int32_t hidden, float eps, int32_t dtype, int32_t rank, int32_t world,
                                         int32_t all_ranks, uint32_t polls, int32_t* err, void* stream) {
  using namespace seb;
  clear_error();
  SEB_CHECK_ARG(dtype == SEB_BF16 || dtype == SEB_F16, "seb_allreduce_add_rmsnorm: bf16 or fp16 required (dtype %d)",
                dtype);
  SEB_CHECK_ARG(world >= 1 && world <= SEB_MAX_PEERS, "seb_allreduce_add_rmsnorm: world %d outside [1, %d]", world,
                SEB_MAX_PEERS);
  SEB_CHECK_ARG(all_ranks ? rank == 0 : (rank >= 0 && rank < world),
                "seb_allreduce_add_rmsnorm: rank %d (world %d, all_ranks %d)", rank, world, all_ranks);
  SEB_CHECK_ARG(n_tokens >= 0 && hidden > 0 && hidden % 8 == 0 && hidden <= 32 * 1024,
                "seb_allreduce_add_rmsnorm: hidden %d must be a multiple of 8 up to 32768", hidden);
  SEB_CHECK_ARG(partial && x && out && flags && weight, "seb_allreduce_add_rmsnorm: NULL pointer argument");
  SEB_CHECK_ARG(aligned(weight, 16), "seb_allreduce_add_rmsnorm: weight must be 16-byte aligned");
  PeerNormParams p{};
  for (int q = 0; q < world; ++q) {
    SEB_CHECK_ARG(partial[q] && x[q] && out[q] && flags[q], "seb_allreduce_add_rmsnorm: NULL buffer of rank %d", q);
    SEB_CHECK_ARG(aligned(partial[q], 16) && aligned(x[q], 16) && aligned(out[q], 16) && aligned(flags[q], 16),
                  "seb_allreduce_add_rmsnorm: buffers of rank %d must be 16-byte aligned", q);
    p.partial[q] = partial[q];
    p.x[q] = x[q];
    p.out[q] = out[q];
    p.flags[q] = static_cast<uint32_t*>(flags[q]);
  }
  p.w = weight;
  p.tokens = n_tokens;
  p.hidden = hidden;
  p.eps = eps;
  p.rank = rank;
  p.world = world;
  p.polls = polls ? polls : kDefaultPolls;
  p.err = err;
  const auto s = static_cast<cudaStream_t>(stream);
  // thread count as in seb_add_rmsnorm, so both round and reduce alike
  if (dtype == SEB_BF16)
    return hidden <= 8192 ? launch_peer_norm<__nv_bfloat16, 256>(p, all_ranks, s)
                          : launch_peer_norm<__nv_bfloat16, 1024>(p, all_ranks, s);
  return hidden <= 8192 ? launch_peer_norm<__half, 256>(p, all_ranks, s)
                        : launch_peer_norm<__half, 1024>(p, all_ranks, s);
}
