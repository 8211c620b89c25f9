// Library-wide C ABI helpers: status strings, error detail, launch counter.
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace sg {

namespace {
thread_local char g_last_error[512] = "";
std::atomic<uint64_t> g_launches{0};
std::mutex g_sm_mutex;
std::vector<int> g_sm_counts;
}  // namespace

void set_error(const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
  va_end(args);
}

void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool enabled = [] {
    const char* v = getenv("SG_PDL");
    return v == nullptr || v[0] != '0';
  }();
  return enabled;
}

L2Window& l2_window() {
  static thread_local L2Window w;
  return w;
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(g_sm_mutex);
  if (static_cast<int>(g_sm_counts.size()) <= dev) g_sm_counts.resize(dev + 1, 0);
  if (g_sm_counts[dev] == 0) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    g_sm_counts[dev] = sms;
  }
  return g_sm_counts[dev];
}

}  // namespace sg

extern "C" const char* sg_status_string(int status) {
  switch (status) {
    case SG_OK: return "ok";
    case SG_ERR_INVALID_ARGUMENT: return "invalid argument";
    case SG_ERR_CUDA: return "CUDA error";
    case SG_ERR_TREE: return "invalid tree metadata";
    case SG_ERR_PROBABILITY: return "invalid target probabilities";
    case SG_ERR_CAPACITY: return "persistent request KV capacity exhausted";
    case SG_ERR_UNSUPPORTED: return "unsupported shape";
    case SG_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

extern "C" const char* sg_last_error(void) { return sg::g_last_error; }

extern "C" int sg_version(void) { return 1; }

extern "C" uint64_t sg_launch_count(void) { return sg::g_launches.load(std::memory_order_relaxed); }
