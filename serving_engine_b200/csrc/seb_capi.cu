// Library-wide C ABI pieces: version, status strings, per-thread error message.
#include "seb_common.cuh"

#include <mutex>

namespace seb {

static thread_local char g_last_error[512] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_last_error[0] = 0; }

int num_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

}  // namespace seb

extern "C" {

const char* seb_version(void) { return "serving_engine_b200 0.1.0 (sm_100a)"; }

const char* seb_status_string(int status) {
  switch (status) {
    case SEB_OK: return "ok";
    case SEB_EINVAL: return "invalid argument";
    case SEB_EUNSUPPORTED: return "unsupported shape or dtype";
    case SEB_ECUDA: return "CUDA error";
    case SEB_EWORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

const char* seb_last_error(void) { return seb::g_last_error; }

}  // extern "C"

// ------------------------------------------------------------ failure self-test
namespace seb {
namespace {

// Waits on an mbarrier that nothing ever arrives on, through the same bounded
// wait every kernel of the library uses, and reports the timeout in the error
// word: the wait gives up after `polls` polls and the kernel returns normally.
__global__ void bounded_wait_selftest_kernel(uint32_t polls, int32_t* err) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait_bounded(b, 0, polls)) atomic_or_err(err, SEB_ERRBIT_TIMEOUT);
}

}  // namespace
}  // namespace seb

extern "C" int seb_selftest_bounded_wait(uint32_t polls, int32_t* err, void* stream) {
  using namespace seb;
  clear_error();
  SEB_CHECK_ARG(err != nullptr, "seb_selftest_bounded_wait: err must point to a device int32");
  SEB_CHECK_ARG(polls > 0 && polls <= (1u << 20), "seb_selftest_bounded_wait: polls must be in [1, 2^20]");
  bounded_wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(polls, err);
  return launch_status("bounded_wait_selftest_kernel");
}
