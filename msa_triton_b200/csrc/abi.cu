// Library-wide ABI helpers: version string and per-thread error messages.
#include "common.cuh"

#include <atomic>
#include <map>
#include <mutex>
#include <vector>

namespace msa {
namespace {
thread_local char g_last_error[1024] = "";
std::atomic<uint64_t> g_launches{0};
}

void count_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

namespace {
struct TimedLaunch {
  cudaEvent_t start, end;
  std::string name;
};
std::mutex g_timing_mu;
std::atomic<bool> g_timing_on{false};
std::vector<TimedLaunch> g_timed;                               // finished pairs, in launch order
std::map<int, std::pair<cudaEvent_t, cudaEvent_t>> g_open;     // slot -> pair whose end is not recorded yet
int g_next_slot = 0;
std::vector<cudaEvent_t> g_event_pool;                          // events reused across reads

cudaEvent_t take_event() {
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}
}  // namespace

int timing_begin(cudaStream_t st) {
  if (!g_timing_on.load(std::memory_order_relaxed)) return -1;
  std::lock_guard<std::mutex> lock(g_timing_mu);
  cudaEvent_t a = take_event(), b = take_event();
  if (!a || !b || cudaEventRecord(a, st) != cudaSuccess) {
    if (a) g_event_pool.push_back(a);
    if (b) g_event_pool.push_back(b);
    return -1;
  }
  const int slot = g_next_slot++;
  g_open[slot] = {a, b};
  return slot;
}

void timing_end(const char* name, int slot, cudaStream_t st) {
  if (slot < 0) return;
  std::lock_guard<std::mutex> lock(g_timing_mu);
  auto it = g_open.find(slot);
  if (it == g_open.end()) return;
  cudaEventRecord(it->second.second, st);
  g_timed.push_back(TimedLaunch{it->second.first, it->second.second, name});
  g_open.erase(it);
}

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

extern "C" int msa_timing_enable(int on) {
  std::lock_guard<std::mutex> lock(msa::g_timing_mu);
  msa::g_timing_on.store(on != 0);
  return MSA_OK;
}

extern "C" int msa_timing_read(const char* kernel, double* total_ms, int64_t* launches) {
  MSA_CHECK_ARG(kernel && total_ms && launches, "msa_timing_read: null argument");
  std::lock_guard<std::mutex> lock(msa::g_timing_mu);
  double sum = 0.0;
  int64_t n = 0;
  std::vector<msa::TimedLaunch> keep;
  for (auto& t : msa::g_timed) {
    if (t.name != kernel) {
      keep.push_back(t);
      continue;
    }
    MSA_CUDA_RETURN(cudaEventSynchronize(t.end));
    float ms = 0.f;
    MSA_CUDA_RETURN(cudaEventElapsedTime(&ms, t.start, t.end));
    sum += ms;
    ++n;
    msa::g_event_pool.push_back(t.start);
    msa::g_event_pool.push_back(t.end);
  }
  msa::g_timed.swap(keep);
  *total_ms = sum;
  *launches = n;
  return MSA_OK;
}
