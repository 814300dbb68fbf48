// Library-wide ABI helpers: version string and per-thread error messages.
#include "common.cuh"

#include <atomic>

namespace msa {
namespace {
thread_local char g_last_error[1024] = "";
std::atomic<uint64_t> g_launches{0};
}

void count_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}
}  // namespace msa

extern "C" const char* msa_version(void) { return "msa_b200 0.1 (sm_100a)"; }

extern "C" const char* msa_last_error(void) { return msa::g_last_error; }

extern "C" uint64_t msa_kernel_launches(void) { return msa::g_launches.load(std::memory_order_relaxed); }
