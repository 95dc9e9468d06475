// Shared host/device helpers of the invokerl_b200 kernels: error reporting across the C ABI,
// launch checks, bf16 conversion and block reductions.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <math.h>

#include "invokerl_b200.h"

namespace ikrl {

// Thread-local last-error buffer behind ikrl_last_error().
void set_error(const char* fmt, ...);
void clear_error();

// Validate one launch: sticky or launch errors become IKRL_ERR_CUDA with the kernel's name.
int check_launch(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Current value of a process-wide launch knob (IKRL_TUNE_*; ikrl_set_tuning).
int64_t tuning(int knob);

constexpr int kNumSMs = 148;  // B200: 2 dies x 74 SMs

}  // namespace ikrl

#define IKRL_REQUIRE(cond, code, ...)        \
  do {                                       \
    if (!(cond)) {                           \
      ::ikrl::set_error(__VA_ARGS__);        \
      return (code);                         \
    }                                        \
  } while (0)

#define IKRL_CUDA(call)                                                              \
  do {                                                                               \
    cudaError_t e__ = (call);                                                        \
    if (e__ != cudaSuccess) {                                                        \
      ::ikrl::set_error("%s failed: %s", #call, cudaGetErrorString(e__));          \
      return IKRL_ERR_CUDA;                                                          \
    }                                                                                \
  } while (0)

namespace ikrl {

// ---- device helpers ----------------------------------------------------------------------

__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ uint16_t f32_to_bf16_rn(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// torch.clamp(x, min=lo): NaN stays NaN (fmaxf would drop it).
__device__ __forceinline__ float clamp_min_nan(float x, float lo) { return x != x ? x : fmaxf(x, lo); }
__device__ __forceinline__ double clamp_min_nan(double x, double lo) { return x != x ? x : fmax(x, lo); }

// 2^x on the MUFU unit (PTX ex2.approx.ftz.f32).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Programmatic dependent launch (sm_90+): a kernel launched with
// cudaLaunchAttributeProgrammaticStreamSerialization may be scheduled while the previous kernel
// of its stream still runs; griddep_wait() blocks until that kernel has finished and its writes
// are visible (a no-op for an ordinary launch).  griddep_launch_dependents() lets the next such
// kernel be scheduled once every block of this grid has called it or exited.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum of NV values per thread; every thread gets the totals.  `scratch` holds
// NV * 32 entries.  Fixed reduction order -> bitwise reproducible.
template <typename T, int NV>
__device__ __forceinline__ void block_sum(T (&v)[NV], T* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] = warp_sum(v[i]);
  __syncthreads();
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < NV; ++i) scratch[i * 32 + warp] = v[i];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    T t = lane < nwarps ? scratch[i * 32 + lane] : T(0);
    v[i] = warp_sum(t);
  }
  __syncthreads();
}

}  // namespace ikrl
