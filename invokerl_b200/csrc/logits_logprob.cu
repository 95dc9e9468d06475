// K2: materialised logits -> per-token log-prob, forward and backward.
//
// Replaces -F.cross_entropy(logits, targets, reduction="none") and its autograd in
// invokerl/policy.py:100-104 (the FSDP branch, which materialises [B, T-1, V] logits) and
// :151-155 (the one-shot branch).  The op is HBM-bound: the forward reads each bf16 logit once,
// the backward reads the logits of rows with a non-zero upstream gradient and writes dlogits.
//
// Layout: one CTA per row; 16-byte vector loads; each thread keeps an online (max, sum-exp)
// pair over its strided slice, combined by warp shuffles and one shared-memory step.  The
// target logit is gathered with one scalar load (bit-exact), so log p = x[t] - lse.
#include "common.cuh"

namespace ikrl {
namespace {

constexpr int kRowThreads = 512;
constexpr int kUnroll = 4;  // 16-byte vectors in flight per thread per iteration

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ void st_stream(uint4* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Online update of (m, s) with 8 values held as 4 packed bf16 pairs; all math in the log2 domain.
__device__ __forceinline__ void online8(const uint4& v, float& m, float& s) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float x[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) { x[2 * k] = bf16lo(w[k]) * kLog2e; x[2 * k + 1] = bf16hi(w[k]) * kLog2e; }
  float mx = x[0];
#pragma unroll
  for (int k = 1; k < 8; ++k) mx = fmaxf(mx, x[k]);
  if (mx > m) {
    s *= fast_exp2(m - mx);
    m = mx;
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) s += fast_exp2(x[k] - m);
}

__device__ __forceinline__ void combine(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) { s = 0.f; m = mm; return; }
  s = s * fast_exp2(m - mm) + s2 * fast_exp2(m2 - mm);
  m = mm;
}

// Block-wide (max, sum) combine; returns lse (natural log) to every thread.
__device__ __forceinline__ float block_lse(float m, float s) {
  __shared__ float sm[32], ss[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    combine(m, s, m2, s2);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { sm[warp] = m; ss[warp] = s; }
  __syncthreads();
  const int nw = blockDim.x >> 5;
  m = lane < nw ? sm[lane] : -INFINITY;
  s = lane < nw ? ss[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    combine(m, s, m2, s2);
  }
  // m, s are in the log2 domain: lse = (m + log2 s) * ln2
  return (m + log2f(s)) * kLn2;
}

__global__ void __launch_bounds__(kRowThreads) logprob_fwd_kernel(
    const uint16_t* __restrict__ logits, int64_t ld, const int64_t* __restrict__ ids, int V,
    float* __restrict__ logp, float* __restrict__ lse_out, float* __restrict__ tgt_out, int vec_ok) {
  const int64_t row = blockIdx.x;
  const uint16_t* x = logits + row * ld;
  float m = -INFINITY, s = 0.f;
  int tail0 = 0;
  if (vec_ok) {
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    const int nv = V >> 3;
    int i = threadIdx.x;
    for (; i + (kUnroll - 1) * kRowThreads < nv; i += kUnroll * kRowThreads) {
      uint4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) v[u] = ld_stream(xv + i + u * kRowThreads);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) online8(v[u], m, s);
    }
    for (; i < nv; i += kRowThreads) online8(ld_stream(xv + i), m, s);
    tail0 = nv << 3;
  }
  for (int j = tail0 + threadIdx.x; j < V; j += kRowThreads) {
    const float v = bf16_to_f32(x[j]) * kLog2e;
    if (v > m) { s *= fast_exp2(m - v); m = v; }
    s += fast_exp2(v - m);
  }
  const float lse = block_lse(m, s);
  if (threadIdx.x == 0) {
    const int64_t t = ids[row];
    float tl, lp;
    if (t == -100) {  // F.cross_entropy ignore_index: loss 0, so -loss is -0.0
      tl = 0.f;
      lp = -0.f;
    } else if (t < 0 || t >= V) {
      tl = lp = __int_as_float(0x7fc00000);
    } else {
      tl = bf16_to_f32(x[t]);
      lp = tl - lse;
    }
    logp[row] = lp;
    lse_out[row] = lse;
    if (tgt_out) tgt_out[row] = tl;
  }
}

__device__ __forceinline__ uint4 dlogits8(const uint4& v, float lse2, float g, int col0, int64_t t) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float p0 = fast_exp2(fmaf(bf16lo(w[k]), kLog2e, -lse2));
    const float p1 = fast_exp2(fmaf(bf16hi(w[k]), kLog2e, -lse2));
    const float d0 = g * (((col0 + 2 * k) == t ? 1.f : 0.f) - p0);
    const float d1 = g * (((col0 + 2 * k + 1) == t ? 1.f : 0.f) - p1);
    o[k] = pack_bf16x2(d0, d1);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void __launch_bounds__(kRowThreads) logprob_bwd_kernel(
    const uint16_t* __restrict__ logits, int64_t ld, const int64_t* __restrict__ ids,
    const float* __restrict__ lse, const float* __restrict__ dlogp, int V, uint16_t* __restrict__ dx,
    int64_t ld_out, int vec_ok) {
  const int64_t row = blockIdx.x;
  const uint16_t* x = logits + row * ld;
  uint16_t* y = dx + row * ld_out;
  const float g0 = dlogp[row];
  const int64_t t = ids[row];
  const bool skip = (g0 == 0.f) || (t == -100);
  const float g = skip ? 0.f : g0;
  const float lse2 = lse[row] * kLog2e;
  int tail0 = 0;
  if (vec_ok) {
    const int nv = V >> 3;
    uint4* yv = reinterpret_cast<uint4*>(y);
    if (skip) {
      const uint4 z = make_uint4(0, 0, 0, 0);
      for (int i = threadIdx.x; i < nv; i += kRowThreads) st_stream(yv + i, z);
    } else {
      const uint4* xv = reinterpret_cast<const uint4*>(x);
      int i = threadIdx.x;
      for (; i + (kUnroll - 1) * kRowThreads < nv; i += kUnroll * kRowThreads) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) v[u] = ld_stream(xv + i + u * kRowThreads);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) st_stream(yv + i + u * kRowThreads, dlogits8(v[u], lse2, g, (i + u * kRowThreads) << 3, t));
      }
      for (; i < nv; i += kRowThreads) st_stream(yv + i, dlogits8(ld_stream(xv + i), lse2, g, i << 3, t));
    }
    tail0 = nv << 3;
  }
  for (int j = tail0 + threadIdx.x; j < V; j += kRowThreads) {
    float d = 0.f;
    if (!skip) {
      const float p = fast_exp2(fmaf(bf16_to_f32(x[j]), kLog2e, -lse2));
      d = g * ((j == t ? 1.f : 0.f) - p);
    }
    y[j] = f32_to_bf16_rn(d);
  }
}

}  // namespace
}  // namespace ikrl

using namespace ikrl;

extern "C" {

int ikrl_logits_logprob_fwd(const void* logits, int64_t ld, const int64_t* ids, int64_t N, int32_t V,
                            float* logp, float* lse, float* tgt_logit, void* stream) {
  clear_error();
  IKRL_REQUIRE(N >= 0 && V > 0 && ld >= V, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_logits_logprob_fwd: bad sizes N=%lld V=%d ld=%lld", (long long)N, V, (long long)ld);
  if (N == 0) return IKRL_OK;
  IKRL_REQUIRE(logits && ids && logp && lse, IKRL_ERR_INVALID_ARGUMENT, "ikrl_logits_logprob_fwd: null pointer");
  IKRL_REQUIRE(N <= 0x7fffffffLL, IKRL_ERR_UNSUPPORTED, "ikrl_logits_logprob_fwd: N=%lld too large", (long long)N);
  const int vec_ok = ((reinterpret_cast<uintptr_t>(logits) & 15) == 0) && (ld % 8 == 0);
  logprob_fwd_kernel<<<(unsigned)N, kRowThreads, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint16_t*>(logits), ld, ids, V, logp, lse, tgt_logit, vec_ok);
  return check_launch("logprob_fwd_kernel");
}

int ikrl_logits_logprob_bwd(const void* logits, int64_t ld, const int64_t* ids, const float* lse,
                            const float* dlogp, int64_t N, int32_t V, void* dlogits, int64_t ld_out, void* stream) {
  clear_error();
  IKRL_REQUIRE(N >= 0 && V > 0 && ld >= V && ld_out >= V, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_logits_logprob_bwd: bad sizes N=%lld V=%d ld=%lld ld_out=%lld", (long long)N, V,
               (long long)ld, (long long)ld_out);
  if (N == 0) return IKRL_OK;
  IKRL_REQUIRE(logits && ids && lse && dlogp && dlogits, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_logits_logprob_bwd: null pointer");
  IKRL_REQUIRE(N <= 0x7fffffffLL, IKRL_ERR_UNSUPPORTED, "ikrl_logits_logprob_bwd: N=%lld too large", (long long)N);
  const int vec_ok = ((reinterpret_cast<uintptr_t>(logits) & 15) == 0) && (ld % 8 == 0) &&
                     ((reinterpret_cast<uintptr_t>(dlogits) & 15) == 0) && (ld_out % 8 == 0);
  logprob_bwd_kernel<<<(unsigned)N, kRowThreads, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint16_t*>(logits), ld, ids, lse, dlogp, V, reinterpret_cast<uint16_t*>(dlogits),
      ld_out, vec_ok);
  return check_launch("logprob_bwd_kernel");
}

}  // extern "C"
