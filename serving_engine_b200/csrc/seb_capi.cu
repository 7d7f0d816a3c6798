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
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
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
