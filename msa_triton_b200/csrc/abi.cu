// Library-wide ABI helpers: version string and per-thread error messages.
#include "common.cuh"

#include <algorithm>
#include <atomic>
#include <cstring>
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

// ---------------------------------------------------------------- small host reads
namespace msa {
namespace {

__global__ void read_i32_kernel(const int32_t* __restrict__ src, int64_t n, int32_t* __restrict__ dst) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

__global__ void block_prefix_kernel(const int32_t* __restrict__ cu, int nseq, int block, int32_t* __restrict__ cbl) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  int32_t acc = 0;
  cbl[0] = 0;
  for (int s = 0; s < nseq; ++s) {
    const int64_t len = (int64_t)cu[s + 1] - cu[s];
    acc += (int32_t)((len + block - 1) / block);
    cbl[s + 1] = acc;
  }
}

// Per-device mapped pinned staging buffer for msa_read_i32.
struct Staging {
  int32_t* host = nullptr;
  int64_t cap = 0;
  cudaEvent_t done = nullptr;
};
std::mutex g_stage_mu;
std::map<int, Staging> g_stage;

}  // namespace
}  // namespace msa

extern "C" int msa_read_i32(const int32_t* src, int64_t n, int32_t* dst, void* stream) {
  MSA_CHECK_ARG(n >= 0 && (n == 0 || (src && dst)), "msa_read_i32: bad arguments");
  if (n == 0) return MSA_OK;
  int dev = 0;
  MSA_CUDA_RETURN(cudaGetDevice(&dev));
  cudaStream_t st = msa::as_stream(stream);
  std::lock_guard<std::mutex> lock(msa::g_stage_mu);
  msa::Staging& s = msa::g_stage[dev];
  if (s.cap < n) {
    if (s.host) MSA_CUDA_RETURN(cudaFreeHost(s.host));
    s.host = nullptr;
    s.cap = 0;
    const int64_t cap = std::max<int64_t>(n, 1024);
    MSA_CUDA_RETURN(cudaHostAlloc(reinterpret_cast<void**>(&s.host), sizeof(int32_t) * cap,
                                  cudaHostAllocMapped | cudaHostAllocPortable));
    s.cap = cap;
  }
  if (!s.done) MSA_CUDA_RETURN(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming));
  int32_t* mapped = nullptr;
  MSA_CUDA_RETURN(cudaHostGetDevicePointer(reinterpret_cast<void**>(&mapped), s.host, 0));
  msa::read_i32_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 1024), 256, 0, st>>>(src, n, mapped);
  msa::count_launches(1);
  if (int e = msa::launch_status("read_i32")) return e;
  MSA_CUDA_RETURN(cudaEventRecord(s.done, st));
  MSA_CUDA_RETURN(cudaEventSynchronize(s.done));
  std::memcpy(dst, s.host, sizeof(int32_t) * n);
  return MSA_OK;
}

extern "C" int msa_block_prefix(const int32_t* cu_seqlens, int32_t nseq, int32_t block_size, int32_t* cu_block_lens,
                                void* stream) {
  MSA_CHECK_ARG(nseq >= 0 && block_size > 0 && cu_seqlens && cu_block_lens, "msa_block_prefix: bad arguments");
  msa::block_prefix_kernel<<<1, 32, 0, msa::as_stream(stream)>>>(cu_seqlens, nseq, block_size, cu_block_lens);
  msa::count_launches(1);
  return msa::launch_status("block_prefix");
}
