// Error plumbing of the C ABI: a thread-local message behind ikrl_last_error().
#include "common.cuh"

#include <atomic>

namespace ikrl {

static std::atomic<unsigned long long> g_launches{0};

static thread_local char g_last_error[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_last_error[0] = 0; }

int check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return IKRL_ERR_CUDA;
  }
  return IKRL_OK;
}

}  // namespace ikrl

extern "C" {

const char* ikrl_last_error(void) { return ikrl::g_last_error; }

int ikrl_abi_version(void) { return 1; }

unsigned long long ikrl_launch_count(void) { return ikrl::g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
