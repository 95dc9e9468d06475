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

namespace {

// Default, lowest and highest value of each knob of ikrl_set_tuning, indexed by IKRL_TUNE_*.
struct KnobSpec {
  int64_t def, lo, hi;
};
constexpr KnobSpec kKnobs[IKRL_TUNE_COUNT] = {
    {1, 0, 1},          // IKRL_TUNE_CTA_PAIRS
    {1, 0, 1},          // IKRL_TUNE_SKIP_ZERO_ROWS
    {-1, -1, 2},        // IKRL_TUNE_WIDE
    {1, 0, 1},          // IKRL_TUNE_PERSISTENT
    {-1, -1, 15},       // IKRL_TUNE_PACE
    {128, 1, 1 << 20},  // IKRL_TUNE_PACE_KB
    {1, 0, 64},         // IKRL_TUNE_PACE_LAG
    {1, 0, 1},          // IKRL_TUNE_BALANCE_SPLITS
    {-1, -1, 22},       // IKRL_TUNE_L2_POLICY
    {0, 0, 1024},       // IKRL_TUNE_L2_BUDGET_MB
    {1, 0, 2},          // IKRL_TUNE_LOSS_KERNEL
    {128, 1, 1 << 20},  // IKRL_TUNE_PACE_KB_LONG
    {4, 0, 4},          // IKRL_TUNE_SPLIT_TAIL
    {-1, -1, 16},       // IKRL_TUNE_DH_SPLIT_K
};

struct Knobs {
  std::atomic<int64_t> v[IKRL_TUNE_COUNT];
  Knobs() {
    for (int i = 0; i < IKRL_TUNE_COUNT; ++i) v[i].store(kKnobs[i].def, std::memory_order_relaxed);
  }
};

Knobs& knobs() {
  static Knobs k;
  return k;
}

}  // namespace

int64_t tuning(int knob) { return knobs().v[knob].load(std::memory_order_relaxed); }

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

int ikrl_set_tuning(int32_t knob, int64_t value, int64_t* previous) {
  using namespace ikrl;
  clear_error();
  IKRL_REQUIRE(knob >= 0 && knob < IKRL_TUNE_COUNT, IKRL_ERR_INVALID_ARGUMENT, "ikrl_set_tuning: unknown knob %d",
               knob);
  if (value == IKRL_TUNE_DEFAULT) value = kKnobs[knob].def;
  IKRL_REQUIRE(value >= kKnobs[knob].lo && value <= kKnobs[knob].hi, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_set_tuning: value %lld of knob %d outside [%lld, %lld]", (long long)value, knob,
               (long long)kKnobs[knob].lo, (long long)kKnobs[knob].hi);
  if (knob == IKRL_TUNE_L2_POLICY && value >= 0)
    IKRL_REQUIRE(value / 10 <= 2 && value % 10 <= 2, IKRL_ERR_INVALID_ARGUMENT,
                 "ikrl_set_tuning: L2 policy %lld is not 10*a + b with a, b in 0..2", (long long)value);
  const int64_t prev = knobs().v[knob].exchange(value, std::memory_order_relaxed);
  if (previous) *previous = prev;
  return IKRL_OK;
}

int ikrl_get_tuning(int32_t knob, int64_t* value) {
  using namespace ikrl;
  clear_error();
  IKRL_REQUIRE(knob >= 0 && knob < IKRL_TUNE_COUNT && value, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_get_tuning: unknown knob %d or null output", knob);
  *value = tuning(knob);
  return IKRL_OK;
}

}  // extern "C"
