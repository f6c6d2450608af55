// Library-wide entry points of the C ABI: error text, version, device facts.
#include <stdarg.h>

#include <atomic>

#include "common.cuh"
#include "../../include/cg_b200.h"

namespace cg {

static thread_local char g_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, args);
  va_end(args);
}

static std::atomic<long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace cg

extern "C" {

const char* cg_last_error(void) { return cg::g_error; }

int cg_version(void) { return CG_B200_ABI_VERSION; }

int64_t cg_launch_count(void) { return cg::g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
