// K3: the advantage and loss hooks of invokerl's algorithms as fused, memory-bound kernels.
//
//   group advantages      invokerl/algorithms/grpo.py:46-80, dapo.py:55-88, base.py:86-110
//   clipped-ratio loss    invokerl/algorithms/grpo.py:84-143, dapo.py:90-150, ppo.py:108-184
//   PPO whitening / GAE   invokerl/algorithms/ppo.py:65-106, :123-127
//   SimPO                 invokerl/algorithms/simpo.py:44-90
//
// The reference runs each of these as 6-30 separate ATen launches plus one blocking .item()
// per metric.  Here the per-token work of a loss is one pass over the tokens that also writes
// d loss / d new_lp, and the metrics come out of a fixed-order (reproducible) reduction in the
// same launch; the host reads them with a single copy.
#include "common.cuh"
#include "sm100.cuh"

namespace ikrl {
namespace {

constexpr int kLossThreads = 256;
#ifndef IKRL_LOSS_UNROLL
#define IKRL_LOSS_UNROLL 2
#endif
#ifndef IKRL_LOSS_BLOCKS_PER_SM
#define IKRL_LOSS_BLOCKS_PER_SM 3
#endif
constexpr int kLossUnroll = IKRL_LOSS_UNROLL;
constexpr int kLossBlocksPerSM = IKRL_LOSS_BLOCKS_PER_SM;
constexpr int kLossMaxBlocks = kNumSMs * kLossBlocksPerSM;
constexpr int kTokenSums = 9;  // sums[0..8] are per-token; [9..15] batch-level

__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// torch.min(a, b) forward value (NaN-propagating) and its backward weights (ties split 1/2).
__device__ __forceinline__ void torch_min2(float a, float b, float& v, float& wa, float& wb) {
  if (a < b) { v = a; wa = 1.f; wb = 0.f; }
  else if (b < a) { v = b; wa = 0.f; wb = 1.f; }
  else if (a == b) { v = a; wa = 0.5f; wb = 0.5f; }
  else { v = __int_as_float(0x7fc00000); wa = 1.f; wb = 1.f; }
}
__device__ __forceinline__ void torch_max2(float a, float b, float& v, float& wa, float& wb) {
  if (a > b) { v = a; wa = 1.f; wb = 0.f; }
  else if (b > a) { v = b; wa = 0.f; wb = 1.f; }
  else if (a == b) { v = a; wa = 0.5f; wb = 0.5f; }
  else { v = __int_as_float(0x7fc00000); wa = 1.f; wb = 1.f; }
}
// torch.clamp(x, lo, hi) value (NaN stays NaN) and whether its gradient passes (closed range).
__device__ __forceinline__ float torch_clamp(float x, float lo, float hi) {
  return x != x ? x : fminf(fmaxf(x, lo), hi);
}

// ---------------------------------------------------------------------------------------------
// Advantages
// ---------------------------------------------------------------------------------------------

// mean and unbiased std of G values (double accumulation; G == 1 -> NaN like torch.std).
__device__ inline void group_stats(const float* r, int G, double& mean, double& std_) {
  double s = 0.0;
  for (int j = 0; j < G; ++j) s += r[j];
  mean = s / G;
  double q = 0.0;
  for (int j = 0; j < G; ++j) { double d = r[j] - mean; q += d * d; }
  std_ = G > 1 ? sqrt(q / (G - 1)) : __longlong_as_double(0x7ff8000000000000ll);
}

// out[t] = a * mask[t] over one row; 16 tokens per step when the row is 16-byte aligned.
__device__ __forceinline__ void broadcast_row(float a, const uint8_t* __restrict__ mrow, float* __restrict__ arow,
                                              int T) {
  int t0 = 0;
  if (((reinterpret_cast<uintptr_t>(mrow) & 3) == 0) && ((reinterpret_cast<uintptr_t>(arow) & 15) == 0)) {
    // 4 tokens per thread per step: a 4-byte mask word in, one 16-byte store out; consecutive
    // threads touch consecutive words, so loads and stores coalesce fully.
    const int n4 = T >> 2;
    const uint32_t* m32 = reinterpret_cast<const uint32_t*>(mrow);
    float4* o = reinterpret_cast<float4*>(arow);
    int i = threadIdx.x;
    for (; i + 3 * (int)blockDim.x < n4; i += 4 * blockDim.x) {
      uint32_t w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) w[u] = __ldg(m32 + i + u * blockDim.x);
#pragma unroll
      for (int u = 0; u < 4; ++u)
        o[i + u * blockDim.x] = make_float4(a * ((w[u] & 0xffu) ? 1.f : 0.f), a * ((w[u] & 0xff00u) ? 1.f : 0.f),
                                            a * ((w[u] & 0xff0000u) ? 1.f : 0.f),
                                            a * ((w[u] & 0xff000000u) ? 1.f : 0.f));
    }
    for (; i < n4; i += blockDim.x) {
      const uint32_t w = __ldg(m32 + i);
      o[i] = make_float4(a * ((w & 0xffu) ? 1.f : 0.f), a * ((w & 0xff00u) ? 1.f : 0.f),
                         a * ((w & 0xff0000u) ? 1.f : 0.f), a * ((w & 0xff000000u) ? 1.f : 0.f));
    }
    t0 = n4 << 2;
  }
  for (int t = t0 + threadIdx.x; t < T; t += blockDim.x) arow[t] = a * (mrow[t] ? 1.f : 0.f);
}

__global__ void group_adv_kernel(const float* __restrict__ rewards, const uint8_t* __restrict__ mask,
                                 const uint8_t* __restrict__ truncated, int B, int T, int G,
                                 int filter_zero_var, float overlong_penalty, float* __restrict__ adv,
                                 float* __restrict__ row_adv) {
  griddep_wait();
  griddep_launch_dependents();
  const int b = blockIdx.x;
  __shared__ float s_adv;
  // Touch this row's mask early so its loads overlap the group statistics below.
  if (threadIdx.x * 16 < T) asm volatile("prefetch.global.L2 [%0];" ::"l"(mask + (int64_t)b * T + threadIdx.x * 16));
  if (threadIdx.x == 0) {
    const int g0 = (b / G) * G;
    double mean, sd;
    group_stats(rewards + g0, G, mean, sd);
    const float meanf = (float)mean, sdf = (float)sd;
    float a;
    if (filter_zero_var) {
      const float valid = (sdf > 1e-8f) ? 1.f : 0.f;
      a = ((rewards[b] - meanf) / clamp_min_nan(sdf, 1e-8f)) * valid;
    } else {
      a = (rewards[b] - meanf) / clamp_min_nan(sdf, 1e-8f);
    }
    if (truncated != nullptr && truncated[b]) a = overlong_penalty;
    s_adv = a;
    if (row_adv) row_adv[b] = a;
  }
  __syncthreads();
  broadcast_row(s_adv, mask + (int64_t)b * T, adv + (int64_t)b * T, T);
}

__global__ void broadcast_adv_kernel(const float* __restrict__ rewards, const uint8_t* __restrict__ mask,
                                     int B, int T, float* __restrict__ adv) {
  const int b = blockIdx.x;
  broadcast_row(rewards[b], mask + (int64_t)b * T, adv + (int64_t)b * T, T);
}

// One thread per (group, position): normalise the G token rewards of that column.
__global__ void token_group_adv_kernel(const float* __restrict__ tr, const uint8_t* __restrict__ mask,
                                       int B, int T, int G, float* __restrict__ adv) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t ngroups = B / G;
  if (i >= ngroups * T) return;
  const int64_t g = i / T, t = i % T;
  const float* base = tr + g * G * (int64_t)T + t;
  double s = 0.0;
  for (int j = 0; j < G; ++j) s += base[(int64_t)j * T];
  const double mean = s / G;
  double q = 0.0;
  for (int j = 0; j < G; ++j) { double d = base[(int64_t)j * T] - mean; q += d * d; }
  const float sdf = G > 1 ? (float)sqrt(q / (G - 1)) : __int_as_float(0x7fc00000);
  const float meanf = (float)mean, den = clamp_min_nan(sdf, 1e-8f);
  for (int j = 0; j < G; ++j) {
    const int64_t o = (g * G + j) * (int64_t)T + t;
    adv[o] = ((tr[o] - meanf) / den) * (mask[o] ? 1.f : 0.f);
  }
}

__global__ void mask_count_kernel(const uint8_t* __restrict__ mask, int64_t n,
                                  unsigned long long* __restrict__ out) {
  unsigned long long c = 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t n16 = ((reinterpret_cast<uintptr_t>(mask) & 15) == 0) ? n / 16 : 0;
  const uint4* m4 = reinterpret_cast<const uint4*>(mask);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) {
    uint4 v = __ldg(m4 + i);
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      // count non-zero bytes
      uint32_t x = w[k];
      x = (x | (x >> 1) | (x >> 2) | (x >> 3) | (x >> 4) | (x >> 5) | (x >> 6) | (x >> 7)) & 0x01010101u;
      c += __popc(x);
    }
  }
  for (int64_t i = n16 * 16 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    c += mask[i] ? 1 : 0;
  c = warp_sum(c);
  if ((threadIdx.x & 31) == 0 && c) atomicAdd(out, c);
}

// ---- PPO whitening moments (two passes, fixed order) --------------------------------------

__global__ void moments_pass_kernel(const float* __restrict__ x, const uint8_t* __restrict__ mask,
                                    int64_t n, int pass, float* __restrict__ out4,
                                    double* __restrict__ partials, unsigned* __restrict__ ticket) {
  __shared__ double scratch[2 * 32];
  __shared__ bool am_last;
  double v[2] = {0.0, 0.0};
  const double mean = pass == 1 ? (double)out4[0] : 0.0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    if (mask[i]) {
      if (pass == 0) { v[0] += x[i]; v[1] += 1.0; }
      else { double d = (double)x[i] - mean; v[0] += d * d; }
    }
  }
  block_sum<double, 2>(v, scratch);
  if (threadIdx.x == 0) {
    partials[blockIdx.x * 2 + 0] = v[0];
    partials[blockIdx.x * 2 + 1] = v[1];
    __threadfence();
    am_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (am_last && threadIdx.x == 0) {
    __threadfence();
    double a = 0.0, c = 0.0;
    for (unsigned b = 0; b < gridDim.x; ++b) { a += __ldcg(partials + 2 * b); c += __ldcg(partials + 2 * b + 1); }
    if (pass == 0) {
      out4[2] = (float)c;
      out4[0] = c > 0 ? (float)(a / c) : __int_as_float(0x7fc00000);
      out4[3] = c > 1 ? 1.f : 0.f;
    } else {
      const double cnt = out4[2];
      out4[1] = cnt > 1 ? (float)sqrt(a / (cnt - 1)) : __int_as_float(0x7fc00000);
    }
    *ticket = 0;
  }
}

// ---- PPO GAE reverse scan ------------------------------------------------------------------
// x_t = delta_t + c_t * x_{t+1} with c_t = gamma*lambda*mask_t and x_T = 0 (ppo.py:96-104).
// One block per row; each thread owns a contiguous chunk, composes its chunk into one affine
// map, a block scan from the right combines the chunks, and a second sweep writes the values.
constexpr int kGaeThreads = 256;

__global__ void gae_kernel(const float* __restrict__ rewards_b, const float* __restrict__ rewards_bt,
                           const float* __restrict__ values, const uint8_t* __restrict__ mask, int T,
                           float gamma, float lam, float* __restrict__ adv) {
  const int b = blockIdx.x;
  const uint8_t* mrow = mask + (int64_t)b * T;
  const float* vrow = values + (int64_t)b * T;
  float* arow = adv + (int64_t)b * T;
  __shared__ int s_last;
  __shared__ float s_A[kGaeThreads], s_B[kGaeThreads];
  // Last response token of the row (sequence reward placement, ppo.py:91-94).
  if (threadIdx.x == 0) s_last = -1;
  __syncthreads();
  if (rewards_bt == nullptr) {
    int last = -1;
    for (int t = threadIdx.x; t < T; t += blockDim.x) if (mrow[t]) last = max(last, t);
    atomicMax(&s_last, last);
  }
  __syncthreads();
  const int last = s_last;
  const float gl = gamma * lam;
  const int chunk = (T + blockDim.x - 1) / blockDim.x;
  const int t0 = threadIdx.x * chunk, t1 = min(T, t0 + chunk);
  auto reward_at = [&](int t) -> float {
    if (rewards_bt) return rewards_bt[(int64_t)b * T + t];
    return t == last ? rewards_b[b] : 0.f;
  };
  // Compose the chunk: x_{t0} = Bc + Ac * x_{t1}.
  float Ac = 1.f, Bc = 0.f;
  for (int t = t1 - 1; t >= t0; --t) {
    const float nv = (t == T - 1) ? 0.f : vrow[t + 1];
    const float delta = reward_at(t) + gamma * nv - vrow[t];
    const float c = gl * (mrow[t] ? 1.f : 0.f);
    Bc = delta + c * Bc;
    Ac = c * Ac;
  }
  s_A[threadIdx.x] = Ac;
  s_B[threadIdx.x] = Bc;
  __syncthreads();
  // Serial combine of the per-thread maps from the right (256 steps, one thread).
  __shared__ float s_in[kGaeThreads];
  if (threadIdx.x == 0) {
    float x = 0.f;
    for (int k = blockDim.x - 1; k >= 0; --k) {
      s_in[k] = x;  // value x_{t1} entering chunk k
      x = s_B[k] + s_A[k] * x;
    }
  }
  __syncthreads();
  float x = s_in[threadIdx.x];
  for (int t = t1 - 1; t >= t0; --t) {
    const float nv = (t == T - 1) ? 0.f : vrow[t + 1];
    const float delta = reward_at(t) + gamma * nv - vrow[t];
    const float m = mrow[t] ? 1.f : 0.f;
    x = delta + gl * x * m;
    arow[t] = x * m;
  }
}

// ---------------------------------------------------------------------------------------------
// Clipped-ratio loss: one pass, d loss / d lp written in the same pass.
// ---------------------------------------------------------------------------------------------

struct LossArgs {
  const void* new_lp;
  const float* old_lp;
  const float* ref_lp;
  const float* adv;
  const uint8_t* mask;
  const int64_t* ntok;
  const float* whiten;
  const float* values;
  const float* old_values;
  const float* rewards;
  int B, G;
  void* dlp;
  float* dvalues;
  double* partials;  // [grid + 1][IKRL_LOSS_NSUMS]: per-block sums, then the batch-level slot
  double* sums;
  int64_t n;
  ikrl_loss_params p;
};

template <bool BF16>
__device__ __forceinline__ float load_lp(const void* p, int64_t i) {
  if constexpr (BF16) return bf16_to_f32(reinterpret_cast<const uint16_t*>(p)[i]);
  else return reinterpret_cast<const float*>(p)[i];
}
template <bool BF16>
__device__ __forceinline__ void store_lp(void* p, int64_t i, float v) {
  if constexpr (BF16) reinterpret_cast<uint16_t*>(p)[i] = f32_to_bf16_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// Per-token body shared by the scalar and vector paths.  acc[] are the masked sums:
//  0 pl*m  1 kl*m  2 clipped*m  3 0.5*lr^2*m  4 adv (masked select)  5 m  6 lp*m  7 vmax*m
//  8 token_loss*m (GRPO)
template <int FAMILY>
__device__ __forceinline__ float token_step(const LossArgs& a, float lp, float old, float ref,
                                            float adv, uint8_t mk, float inv_n, float wmean,
                                            float wstd, bool whiten_on, float vv, float ov,
                                            float& dval, float (&acc)[kTokenSums]) {
  const ikrl_loss_params& p = a.p;
  const float m = mk ? 1.f : 0.f;
  if (whiten_on) adv = ((adv - wmean) / (wstd + 1e-8f)) * m;
  const float lr = lp - old;
  // ratio = e^lr as 2^(lr * log2 e) on the MUFU unit: a few ulp, well inside the 1e-4 parity bound.
  const float rho = fast_exp2(lr * kLog2e);
  const float s1 = rho * adv;
  const float rc = torch_clamp(rho, p.ratio_lo, p.ratio_hi);
  const float s2 = rc * adv;
  float mn, w1, w2;
  torch_min2(s1, s2, mn, w1, w2);
  const float pl = -mn;
  const float inb = (rho >= p.ratio_lo && rho <= p.ratio_hi) ? 1.f : 0.f;
  // d pl / d lp  (grad_rho = w1*A + w2*A*inb; exp backward multiplies by rho)
  const float dpl = -((w1 * adv + w2 * (adv * inb)) * rho);

  float kl = 0.f, dkl = 0.f;
  const bool has_kl = (a.ref_lp != nullptr) && (p.kl_type != IKRL_KL_NONE) &&
                      (FAMILY == IKRL_LOSS_GRPO || p.beta > 0.f);
  if (has_kl) {
    const float lrr = ref - lp;
    if (p.kl_type == IKRL_KL_SCHULMAN) {
      const float e = expf(lrr);
      kl = e - lrr - 1.f;
      dkl = 1.f - e;
    } else {
      kl = -lrr;
      dkl = 1.f;
    }
  }
  const float g = m * inv_n;  // d (sum(x*m)/n) / d x
  float dlp;
  acc[0] += pl * m;
  acc[1] += kl * m;
  acc[2] += (fabsf(rho - 1.f) > p.clip_metric_eps ? 1.f : 0.f) * m;
  acc[3] += (0.5f * (lr * lr)) * m;
  if (mk) acc[4] += adv;
  acc[5] += m;
  acc[6] += lp * m;
  if constexpr (FAMILY == IKRL_LOSS_GRPO) {
    const float tl = pl + p.beta * kl;
    acc[8] += tl * m;
    dlp = g * dpl + (g * p.beta) * dkl;
  } else {
    dlp = g * dpl + p.entropy_coef * g;
    if (has_kl) dlp += (p.beta * g) * dkl;
    if (a.values != nullptr) {
      const float ret = adv + ov;
      const float dv = vv - ov;
      const float vclip = ov + torch_clamp(dv, -p.vf_clip_eps, p.vf_clip_eps);
      const float e1 = vv - ret, e2 = vclip - ret;
      const float l1 = e1 * e1, l2 = e2 * e2;
      float vmax, u1, u2;
      torch_max2(l1, l2, vmax, u1, u2);
      acc[7] += vmax * m;
      const float vinb = (dv >= -p.vf_clip_eps && dv <= p.vf_clip_eps) ? 1.f : 0.f;
      const float gv = p.vf_coef * 0.5f * g;
      dval = gv * (u1 * 2.f * e1 + u2 * 2.f * e2 * vinb);
    }
  }
  return dlp;
}

template <bool BF16>
__device__ __forceinline__ void load_lp4(const void* p, int64_t q, float (&x)[4]) {
  if constexpr (BF16) {
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(p) + q);
    x[0] = bf16lo(w.x); x[1] = bf16hi(w.x); x[2] = bf16lo(w.y); x[3] = bf16hi(w.y);
  } else {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p) + q);
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  }
}
template <bool BF16>
__device__ __forceinline__ void store_lp4(void* p, int64_t q, const float (&x)[4]) {
  if constexpr (BF16) {
    reinterpret_cast<uint2*>(p)[q] = make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
  } else {
    reinterpret_cast<float4*>(p)[q] = make_float4(x[0], x[1], x[2], x[3]);
  }
}
__device__ __forceinline__ void ld4(const float* p, int64_t q, float (&x)[4]) {
  const float4 v = __ldg(reinterpret_cast<const float4*>(p) + q);
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}

// The loss kernels run one block more than they give tokens to: block 0 computes the batch-level
// reward terms (they take a few µs of dependent loads) while blocks 1.. process the tokens, so no
// token block finishes late.  With a one-block grid, block 0 does both.
struct TokenGrid {
  int tb;  // this block's index among the token blocks (-1: the batch-terms block)
  int nb;  // number of token blocks
};
__device__ __forceinline__ TokenGrid token_grid() {
  const int tok0 = gridDim.x > 1 ? 1 : 0;
  return {(int)blockIdx.x - tok0, (int)gridDim.x - tok0};
}
__host__ __device__ inline int token_blocks(int grid) { return grid > 1 ? grid - 1 : 1; }

// Per-block sums -> partials[slot] (fixed order: float warp sums, then a double sum over the
// warps).  The token blocks' sums are combined afterwards, in a fixed order, by
// loss_sums_reduce_kernel (a separate launch, so no block waits on the others and no counter has
// to be reset between calls).
__device__ __forceinline__ void write_block_sums(const LossArgs& a, const float (&v)[kTokenSums], double* scratch,
                                                 int slot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  float w[kTokenSums];
#pragma unroll
  for (int i = 0; i < kTokenSums; ++i) w[i] = warp_sum(v[i]);
  __syncthreads();  // scratch may still be read by an earlier block-wide reduction
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < kTokenSums; ++i) scratch[i * 32 + warp] = (double)w[i];
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int i = 0; i < kTokenSums; ++i) {
      double t = lane < nw ? scratch[i * 32 + lane] : 0.0;
      t = warp_sum(t);
      if (lane == 0) a.partials[(int64_t)slot * IKRL_LOSS_NSUMS + i] = t;
    }
  }
}

// Batch-level terms: rewards.sum() (for rewards.mean()) and the zero-variance group count
// (dapo.py:132-135), into the slot after the nb token blocks' partials.
__device__ __forceinline__ void write_batch_terms(const LossArgs& a, double* scratch, int nb) {
  double r[2] = {0.0, 0.0};
  for (int b = threadIdx.x; b < a.B; b += blockDim.x) r[0] += a.rewards[b];
  if (a.G > 0) {
    for (int g = threadIdx.x; g < a.B / a.G; g += blockDim.x) {
      double mean, sd;
      group_stats(a.rewards + g * a.G, a.G, mean, sd);
      if ((float)sd < 1e-8f) r[1] += 1.0;
    }
  }
  block_sum<double, 2>(r, scratch);
  if (threadIdx.x == 0) {
    a.partials[(int64_t)nb * IKRL_LOSS_NSUMS + 0] = r[0];
    a.partials[(int64_t)nb * IKRL_LOSS_NSUMS + 1] = r[1];
  }
}

// sums[0..8] = fixed-order sum of the nblocks per-block partials (thread i takes blocks i,
// i + 256, ..., then the block tree combines the threads); sums[9..12] the batch-level terms.
// derive_token_loss: sums[8] = sums[0] + beta * sums[1] (the lean GRPO kernels leave it out).
__global__ void __launch_bounds__(256) loss_sums_reduce_kernel(const double* __restrict__ partials, int nblocks,
                                                               int derive_token_loss, float beta, int B, int G,
                                                               double* __restrict__ sums) {
  __shared__ double scratch[IKRL_LOSS_NSUMS * 32];
  // Launched as a programmatic dependent of the loss kernel: it may start while that kernel runs
  // and waits here until it has completed and its partials are visible.
  griddep_wait();
  griddep_launch_dependents();
  double t[kTokenSums];
#pragma unroll
  for (int i = 0; i < kTokenSums; ++i) t[i] = 0.0;
  for (int b = threadIdx.x; b < nblocks; b += blockDim.x) {
#pragma unroll
    for (int i = 0; i < kTokenSums; ++i) t[i] += partials[(int64_t)b * IKRL_LOSS_NSUMS + i];
  }
  block_sum<double, kTokenSums>(t, scratch);
  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < kTokenSums; ++i) sums[i] = t[i];
    if (derive_token_loss) sums[8] = t[0] + (double)beta * t[1];
    sums[9] = partials[(int64_t)nblocks * IKRL_LOSS_NSUMS + 0];
    sums[10] = (double)B;
    sums[11] = partials[(int64_t)nblocks * IKRL_LOSS_NSUMS + 1];
    sums[12] = G > 0 ? (double)(B / G) : 0.0;
    sums[13] = sums[14] = sums[15] = 0.0;
  }
}

// VEC: four tokens per thread per step with 16-byte loads (n % 4 == 0, aligned pointers).
template <int FAMILY, bool BF16, bool VEC>
__global__ void __launch_bounds__(kLossThreads, kLossBlocksPerSM) clip_loss_kernel(LossArgs a) {
  __shared__ double scratch[IKRL_LOSS_NSUMS * 32];
  // Inputs may come from the previous kernel of the stream (programmatic dependent launch).
  griddep_wait();
  // Every block has started: the sums-reduce kernel may be scheduled now (it waits for this grid).
  griddep_launch_dependents();
  const TokenGrid tg = token_grid();
  if (blockIdx.x == 0) write_batch_terms(a, scratch, tg.nb);
  if (tg.tb < 0) return;
  float acc[kTokenSums];
#pragma unroll
  for (int i = 0; i < kTokenSums; ++i) acc[i] = 0.f;

  const float inv_n = 1.f / fmaxf((float)(*a.ntok), 1.f);
  const bool whiten_on = a.whiten != nullptr && a.whiten[3] != 0.f;
  const float wmean = whiten_on ? a.whiten[0] : 0.f, wstd = whiten_on ? a.whiten[1] : 0.f;
  const int64_t stride = (int64_t)tg.nb * blockDim.x;
  if constexpr (VEC) {
    // kLossUnroll quads per thread per step, all loads issued before any compute.
    const int64_t nq = a.n >> 2;
    for (int64_t q0 = (int64_t)tg.tb * blockDim.x + threadIdx.x; q0 < nq; q0 += stride * kLossUnroll) {
      float lp[kLossUnroll][4], old[kLossUnroll][4], ref[kLossUnroll][4], adv[kLossUnroll][4];
      float vv[kLossUnroll][4], ov[kLossUnroll][4];
      uint32_t mw[kLossUnroll];
#pragma unroll
      for (int u = 0; u < kLossUnroll; ++u) {
        const int64_t q = q0 + u * stride;
#pragma unroll
        for (int j = 0; j < 4; ++j) { ref[u][j] = 0.f; vv[u][j] = 0.f; ov[u][j] = 0.f; }
        mw[u] = 0;
        if (q < nq) {
          load_lp4<BF16>(a.new_lp, q, lp[u]);
          ld4(a.old_lp, q, old[u]);
          if (a.ref_lp) ld4(a.ref_lp, q, ref[u]);
          ld4(a.adv, q, adv[u]);
          mw[u] = __ldg(reinterpret_cast<const uint32_t*>(a.mask) + q);
          if (a.values) { ld4(a.values, q, vv[u]); ld4(a.old_values, q, ov[u]); }
        }
      }
#pragma unroll
      for (int u = 0; u < kLossUnroll; ++u) {
        const int64_t q = q0 + u * stride;
        if (q >= nq) break;
        float d[4], dv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint8_t mk = (uint8_t)((mw[u] >> (8 * j)) & 0xffu);
          d[j] = token_step<FAMILY>(a, lp[u][j], old[u][j], ref[u][j], adv[u][j], mk, inv_n, wmean, wstd,
                                    whiten_on, vv[u][j], ov[u][j], dv[j], acc);
        }
        if (a.dlp) store_lp4<BF16>(a.dlp, q, d);
        if (a.dvalues) reinterpret_cast<float4*>(a.dvalues)[q] = make_float4(dv[0], dv[1], dv[2], dv[3]);
      }
    }
  } else {
    for (int64_t i = (int64_t)tg.tb * blockDim.x + threadIdx.x; i < a.n; i += stride) {
      const float lp = load_lp<BF16>(a.new_lp, i);
      const float old = __ldg(a.old_lp + i);
      const float ref = a.ref_lp ? __ldg(a.ref_lp + i) : 0.f;
      const float adv = __ldg(a.adv + i);
      const uint8_t mk = __ldg(a.mask + i);
      const float vv = a.values ? __ldg(a.values + i) : 0.f;
      const float ov = a.values ? __ldg(a.old_values + i) : 0.f;
      float dval = 0.f;
      const float d = token_step<FAMILY>(a, lp, old, ref, adv, mk, inv_n, wmean, wstd, whiten_on,
                                         vv, ov, dval, acc);
      if (a.dlp) store_lp<BF16>(a.dlp, i, d);
      if (a.dvalues) a.dvalues[i] = dval;
    }
  }

  write_block_sums(a, acc, scratch, tg.tb);
}

// Masked sums of the lean GRPO / DAPO pass (grpo.py:103-140): policy loss, KL, clip count,
// (lp - old)^2, advantages of masked tokens, token count, lp.
struct GrpoSums {
  float pl = 0.f, kl = 0.f, clip = 0.f, lr2 = 0.f, adv = 0.f, m = 0.f, lp = 0.f;
};

// One token of GRPO / DAPO: accumulates the masked sums and returns d loss / d lp.
// KL: 0 none, 1 k3 (schulman), 2 k1 (simple).
template <int KL>
__device__ __forceinline__ float grpo_token(float x, float o, float r, float A, bool mk, float inv_n, float lo,
                                            float hi, float ceps, float beta, GrpoSums& acc) {
  const float m = mk ? 1.f : 0.f;
  const float lr = x - o;
  // ratio = e^lr as 2^(lr * log2 e) on the MUFU unit: a few ulp, well inside the 1e-4 parity bound.
  const float rho = fast_exp2(lr * kLog2e);
  const float s1 = rho * A;
  const float s2 = torch_clamp(rho, lo, hi) * A;
  float mn, w1, w2;
  torch_min2(s1, s2, mn, w1, w2);
  const float inb = (rho >= lo && rho <= hi) ? 1.f : 0.f;
  const float dpl = -((w1 * A + w2 * (A * inb)) * rho);
  float kl = 0.f, dkl = 0.f;
  if constexpr (KL == 1) {
    const float lrr = r - x;
    const float e = fast_exp2(lrr * kLog2e);
    kl = e - lrr - 1.f;
    dkl = 1.f - e;
  } else if constexpr (KL == 2) {
    kl = -(r - x);
    dkl = 1.f;
  }
  const float g = m * inv_n;
  acc.pl += (-mn) * m;
  acc.kl += kl * m;
  acc.clip += (fabsf(rho - 1.f) > ceps ? 1.f : 0.f) * m;
  acc.lr2 += (lr * lr) * m;
  if (mk) acc.adv += A;
  acc.m += m;
  acc.lp += x * m;
  return g * dpl + (g * beta) * dkl;
}

__device__ __forceinline__ void grpo_finish(const LossArgs& a, const GrpoSums& acc, double* scratch, int slot,
                                            bool aborted = false) {
  float v[kTokenSums] = {acc.pl, acc.kl, acc.clip, 0.5f * acc.lr2, acc.adv, acc.m, acc.lp, 0.f, 0.f};
  if (aborted) v[0] = __int_as_float(0x7fc00000);  // a gave-up wait poisons the loss
  write_block_sums(a, v, scratch, slot);
}

// GRPO / DAPO with no value head and no whitening (grpo.py:84-143, dapo.py:90-150): four tokens
// per thread per step on 16-byte loads, KL form fixed at compile time, and only the sums those
// losses report.  The token loss sum(pl*m) + beta*sum(kl*m) is formed from its two parts after
// the reduction instead of per token.
template <bool BF16, int KL>
__global__ void __launch_bounds__(kLossThreads, kLossBlocksPerSM) grpo_loss_kernel(LossArgs a) {
  __shared__ double scratch[IKRL_LOSS_NSUMS * 32];
  // Inputs may come from the previous kernel of the stream (programmatic dependent launch).
  griddep_wait();
  // Every block has started: the sums-reduce kernel may be scheduled now (it waits for this grid).
  griddep_launch_dependents();
  const TokenGrid tg = token_grid();
  if (blockIdx.x == 0) write_batch_terms(a, scratch, tg.nb);
  if (tg.tb < 0) return;
  GrpoSums acc;
  const float inv_n = 1.f / fmaxf((float)(*a.ntok), 1.f);
  const float lo = a.p.ratio_lo, hi = a.p.ratio_hi, ceps = a.p.clip_metric_eps, beta = a.p.beta;
  const int64_t stride = (int64_t)tg.nb * blockDim.x;
  const int64_t nq = a.n >> 2;
  for (int64_t q0 = (int64_t)tg.tb * blockDim.x + threadIdx.x; q0 < nq; q0 += stride * kLossUnroll) {
    float lp[kLossUnroll][4], old[kLossUnroll][4], ref[kLossUnroll][4], adv[kLossUnroll][4];
    uint32_t mw[kLossUnroll];
#pragma unroll
    for (int u = 0; u < kLossUnroll; ++u) {
      const int64_t q = q0 + u * stride;
      if (q < nq) {
        load_lp4<BF16>(a.new_lp, q, lp[u]);
        ld4(a.old_lp, q, old[u]);
        if constexpr (KL != 0) ld4(a.ref_lp, q, ref[u]);
        ld4(a.adv, q, adv[u]);
        mw[u] = __ldg(reinterpret_cast<const uint32_t*>(a.mask) + q);
      }
    }
#pragma unroll
    for (int u = 0; u < kLossUnroll; ++u) {
      const int64_t q = q0 + u * stride;
      if (q >= nq) break;
      float d[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        d[j] = grpo_token<KL>(lp[u][j], old[u][j], KL != 0 ? ref[u][j] : 0.f, adv[u][j],
                              ((mw[u] >> (8 * j)) & 0xffu) != 0u, inv_n, lo, hi, ceps, beta, acc);
      if (a.dlp) store_lp4<BF16>(a.dlp, q, d);
    }
  }
  grpo_finish(a, acc, scratch, tg.tb);
}

// The same pass with the inputs staged through shared memory by bulk copies (cp.async.bulk,
// completion on an mbarrier): one producer thread keeps kBulkStages tiles of 1024 tokens per
// block in flight, independent of the registers of the 256 consumer threads, which read their
// four tokens of a tile from shared memory.  Tiles are dealt to the blocks round-robin; the one
// partial tile at the end (n % 1024 tokens) is read directly from global memory.
using namespace sm100;

constexpr int kBulkTile = 1024;
constexpr int kBulkStages = 4;
constexpr int kBulkConsumers = 256;
constexpr int kBulkThreads = kBulkConsumers + 32;
constexpr int kBulkBlocksPerSM = 2;

template <bool BF16>
constexpr uint32_t bulk_stage_bytes() {
  return kBulkTile * ((BF16 ? 2 : 4) + 4 + 4 + 4 + 1);
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

template <bool BF16, int KL>
__global__ void __launch_bounds__(kBulkThreads, kBulkBlocksPerSM) grpo_loss_bulk_kernel(LossArgs a) {
  extern __shared__ __align__(128) uint8_t bulk_smem[];
  __shared__ double scratch[IKRL_LOSS_NSUMS * 32];
  __shared__ __align__(8) uint64_t full_bar[kBulkStages], empty_bar[kBulkStages];
  __shared__ int abort_flag, err_word;
  constexpr uint32_t kLpBytes = kBulkTile * (BF16 ? 2 : 4);
  constexpr uint32_t kOffOld = kLpBytes, kOffRef = kOffOld + 4 * kBulkTile, kOffAdv = kOffRef + 4 * kBulkTile,
                     kOffMask = kOffAdv + 4 * kBulkTile;
  constexpr uint32_t kStage = bulk_stage_bytes<BF16>();
  // Inputs may come from the previous kernel of the stream (programmatic dependent launch).
  griddep_wait();
  // Every block has started: the sums-reduce kernel may be scheduled now (it waits for this grid).
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_full = a.n / kBulkTile;
  const int64_t n_tiles = (a.n + kBulkTile - 1) / kBulkTile;
  volatile int* abort_v = &abort_flag;
  int* err = &err_word;

  if (threadIdx.x == 0) {
    for (int st = 0; st < kBulkStages; ++st) {
      mbar_init(smem_u32(&full_bar[st]), 1);
      mbar_init(smem_u32(&empty_bar[st]), kBulkConsumers / 32);
    }
    abort_flag = 0;
    err_word = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const TokenGrid tg = token_grid();
  if (blockIdx.x == 0) write_batch_terms(a, scratch, tg.nb);
  if (tg.tb < 0) return;
  const uint32_t sbase = smem_u32(bulk_smem);
  GrpoSums acc;

  if (warp == kBulkConsumers / 32) {
    // ---- producer ----
    if (lane == 0) {
      int i = 0;
      for (int64_t t = tg.tb; t < n_full; t += tg.nb, ++i) {
        const int st = i % kBulkStages;
        const uint32_t ph = (uint32_t)(i / kBulkStages) & 1u;
        if (!mbar_wait(smem_u32(&empty_bar[st]), ph ^ 1u, abort_v, err, kErrTimeoutProducer)) break;
        const uint32_t fb = smem_u32(&full_bar[st]);
        const uint32_t dst = sbase + st * kStage;
        const int64_t t0 = t * kBulkTile;
        mbar_arrive_expect_tx(fb, KL != 0 ? kStage : kStage - 4 * kBulkTile);
        bulk_g2s(dst, reinterpret_cast<const uint8_t*>(a.new_lp) + t0 * (BF16 ? 2 : 4), kLpBytes, fb);
        bulk_g2s(dst + kOffOld, a.old_lp + t0, 4 * kBulkTile, fb);
        if constexpr (KL != 0) bulk_g2s(dst + kOffRef, a.ref_lp + t0, 4 * kBulkTile, fb);
        bulk_g2s(dst + kOffAdv, a.adv + t0, 4 * kBulkTile, fb);
        bulk_g2s(dst + kOffMask, a.mask + t0, kBulkTile, fb);
      }
      // Copies still in flight after a gave-up wait land before the block leaves.
      if (*abort_v) {
        const int issued = i;
        for (int j = 0; j < kBulkStages && j < issued; ++j) {
          const int k = issued - 1 - j;
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(smem_u32(&full_bar[k % kBulkStages]), (uint32_t)(k / kBulkStages) & 1u)) {
            if (globaltimer() - t0 > kWaitTimeoutNs / 4) break;
          }
        }
      }
    }
  } else {
    // ---- consumers: four tokens each per tile ----
    const float inv_n = 1.f / fmaxf((float)(*a.ntok), 1.f);
    const float lo = a.p.ratio_lo, hi = a.p.ratio_hi, ceps = a.p.clip_metric_eps, beta = a.p.beta;
    int i = 0;
    for (int64_t t = tg.tb; t < n_full; t += tg.nb, ++i) {
      const int st = i % kBulkStages;
      const uint32_t ph = (uint32_t)(i / kBulkStages) & 1u;
      if (!mbar_wait(smem_u32(&full_bar[st]), ph, abort_v, err, kErrTimeoutEpilogue)) break;
      const uint8_t* sp = bulk_smem + st * kStage;
      float x[4], o[4], r[4] = {0.f, 0.f, 0.f, 0.f}, A[4];
      if constexpr (BF16) {
        const uint2 w = reinterpret_cast<const uint2*>(sp)[threadIdx.x];
        x[0] = bf16lo(w.x); x[1] = bf16hi(w.x); x[2] = bf16lo(w.y); x[3] = bf16hi(w.y);
      } else {
        const float4 v = reinterpret_cast<const float4*>(sp)[threadIdx.x];
        x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
      }
      {
        const float4 v = reinterpret_cast<const float4*>(sp + kOffOld)[threadIdx.x];
        o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
      }
      if constexpr (KL != 0) {
        const float4 v = reinterpret_cast<const float4*>(sp + kOffRef)[threadIdx.x];
        r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
      }
      {
        const float4 v = reinterpret_cast<const float4*>(sp + kOffAdv)[threadIdx.x];
        A[0] = v.x; A[1] = v.y; A[2] = v.z; A[3] = v.w;
      }
      const uint32_t mw = reinterpret_cast<const uint32_t*>(sp + kOffMask)[threadIdx.x];
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&empty_bar[st]));  // the tile's smem may be refilled
      float d[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        d[j] = grpo_token<KL>(x[j], o[j], r[j], A[j], ((mw >> (8 * j)) & 0xffu) != 0u, inv_n, lo, hi, ceps, beta,
                              acc);
      if (a.dlp) store_lp4<BF16>(a.dlp, t * (kBulkTile / 4) + threadIdx.x, d);
    }
    // the partial tile, if any, goes to the block that would have been dealt it
    if (n_tiles > n_full && (n_full % tg.nb) == tg.tb && !*abort_v) {
      for (int64_t k = n_full * kBulkTile + threadIdx.x; k < a.n; k += kBulkConsumers) {
        const float x = load_lp<BF16>(a.new_lp, k);
        const float d = grpo_token<KL>(x, a.old_lp[k], KL != 0 ? a.ref_lp[k] : 0.f, a.adv[k], a.mask[k] != 0, inv_n,
                                       lo, hi, ceps, beta, acc);
        if (a.dlp) store_lp<BF16>(a.dlp, k, d);
      }
    }
  }
  __syncthreads();
  grpo_finish(a, acc, scratch, tg.tb, *abort_v != 0);
}

__global__ void clip_loss_finalize_kernel(const double* __restrict__ s, const int64_t* __restrict__ ntok,
                                          ikrl_loss_params p, float* __restrict__ loss_out,
                                          float* __restrict__ metrics) {
  griddep_wait();
  griddep_launch_dependents();
  if (threadIdx.x != 0) return;
  const double n = fmax((double)(float)(*ntok), 1.0);
  const float nf = (float)n;
  double loss;
  const double pl = s[0] / n, kl = s[1] / n, entropy = -s[6] / n;
  if (p.family == IKRL_LOSS_GRPO) {
    loss = (float)(s[8]) / nf;
  } else {
    const float plm = (float)s[0] / nf;
    const float vf = 0.5f * (float)s[7] / nf;
    const float ent = -((float)s[6]) / nf;
    float l = plm + p.vf_coef * vf + (-p.entropy_coef * ent);
    if (p.beta > 0.f) l += p.beta * ((float)s[1] / nf);
    loss = l;
  }
  loss_out[0] = (float)loss;
  metrics[0] = (float)loss;
  metrics[1] = s[10] > 0 ? (float)(s[9] / s[10]) : __int_as_float(0x7fc00000);
  metrics[2] = (float)kl;
  metrics[3] = (float)pl;
  metrics[4] = (float)(s[2] / n);
  metrics[5] = (float)(s[3] / n);
  metrics[6] = s[5] > 0 ? (float)(s[4] / s[5]) : 0.f;
  metrics[7] = (float)entropy;
  metrics[8] = (float)(0.5 * s[7] / n);
  metrics[9] = (float)n;
  metrics[10] = (float)s[11];
  metrics[11] = (float)s[12];
}

template <bool BF16>
__global__ void scale_grad_kernel(void* g, int64_t n, const float* __restrict__ scale) {
  griddep_wait();
  griddep_launch_dependents();
  const float s = *scale;
  if (s == 1.f) return;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    if constexpr (BF16) {
      uint16_t* p = reinterpret_cast<uint16_t*>(g);
      p[i] = f32_to_bf16_rn(bf16_to_f32(p[i]) * s);
    } else {
      float* p = reinterpret_cast<float*>(g);
      p[i] = p[i] * s;
    }
  }
}

// ---- SimPO -----------------------------------------------------------------------------------

template <bool BF16>
__global__ void simpo_rows_kernel(const void* lp, const uint8_t* __restrict__ mask, int T,
                                  float* __restrict__ avg, float* __restrict__ len) {
  __shared__ float scratch[2 * 32];
  const int b = blockIdx.x;
  float v[2] = {0.f, 0.f};
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const int64_t i = (int64_t)b * T + t;
    const float m = mask[i] ? 1.f : 0.f;
    v[0] += load_lp<BF16>(lp, i) * m;
    v[1] += m;
  }
  block_sum<float, 2>(v, scratch);
  if (threadIdx.x == 0) {
    const float l = fmaxf(v[1], 1.f);
    len[b] = l;
    avg[b] = v[0] / l;
  }
}

__device__ __forceinline__ float log_sigmoid(float x) {
  // log(sigmoid(x)) = min(x, 0) - log1p(exp(-|x|))
  return fminf(x, 0.f) - log1pf(expf(-fabsf(x)));
}

__global__ void simpo_pairs_kernel(const float* __restrict__ avg, const float* __restrict__ len,
                                   const float* __restrict__ rewards, int B, float beta, float gamma,
                                   int chosen_first, float* __restrict__ loss_out,
                                   float* __restrict__ metrics, float* __restrict__ row_coef) {
  __shared__ double scratch[6 * 32];
  const int P = B / 2;
  double v[6] = {0, 0, 0, 0, 0, 0};
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const int ic = chosen_first ? 2 * i : 2 * i + 1;
    const int ir = chosen_first ? 2 * i + 1 : 2 * i;
    const float c = avg[ic], r = avg[ir];
    const float margin = beta * (c - r) - gamma;
    v[0] += -log_sigmoid(margin);
    v[1] += c;
    v[2] += r;
    v[3] += (c > r) ? 1.0 : 0.0;
    v[4] += margin;
    // d(-logsigmoid(m))/dm = sigmoid(m) - 1, mean over P pairs
    const float dm = (1.f / (1.f + expf(-margin)) - 1.f) / (float)P;
    row_coef[ic] = beta * dm / len[ic];
    row_coef[ir] = -beta * dm / len[ir];
  }
  for (int b = threadIdx.x; b < B; b += blockDim.x) v[5] += avg[b];
  block_sum<double, 6>(v, scratch);
  if (threadIdx.x == 0) {
    double r = 0.0;
    for (int b = 0; b < B; ++b) r += rewards ? rewards[b] : 0.0;
    const float loss = (float)(v[0] / P);
    loss_out[0] = loss;
    metrics[0] = loss;
    metrics[1] = rewards ? (float)(r / B) : 0.f;
    metrics[2] = (float)(v[1] / P);
    metrics[3] = (float)(v[2] / P);
    metrics[4] = (float)(v[3] / P);
    metrics[5] = (float)(v[4] / P);
    metrics[6] = (float)(v[5] / B);
    metrics[7] = (float)P;
  }
}

template <bool BF16>
__global__ void simpo_bwd_kernel(const float* __restrict__ row_coef, const uint8_t* __restrict__ mask,
                                 int T, const float* __restrict__ scale, void* dlp) {
  const int b = blockIdx.x;
  const float c = row_coef[b] * *scale;
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const int64_t i = (int64_t)b * T + t;
    store_lp<BF16>(dlp, i, c * (mask[i] ? 1.f : 0.f));
  }
}

// ---- DPO -------------------------------------------------------------------------------------
// log_ratio[b] = sum_t (lp - ref) * m  (dpo.py:66-70), then the pairwise sigmoid loss.

template <bool BF16>
__global__ void dpo_rows_kernel(const void* lp, const float* __restrict__ ref, const uint8_t* __restrict__ mask,
                                int T, float* __restrict__ log_ratio) {
  __shared__ float scratch[2 * 32];
  const int b = blockIdx.x;
  float v[2] = {0.f, 0.f};
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const int64_t i = (int64_t)b * T + t;
    const float m = mask[i] ? 1.f : 0.f;
    v[0] += load_lp<BF16>(lp, i) * m;
    v[1] += ref[i] * m;
  }
  block_sum<float, 2>(v, scratch);
  if (threadIdx.x == 0) log_ratio[b] = v[0] - v[1];
}

__global__ void dpo_pairs_kernel(const float* __restrict__ lr, const float* __restrict__ rewards, int B, float beta,
                                 float smoothing, int chosen_first, float* __restrict__ loss_out,
                                 float* __restrict__ metrics, float* __restrict__ row_coef) {
  __shared__ double scratch[5 * 32];
  const int P = B / 2;
  double v[5] = {0, 0, 0, 0, 0};
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const int ic = chosen_first ? 2 * i : 2 * i + 1;
    const int ir = chosen_first ? 2 * i + 1 : 2 * i;
    const float c = lr[ic], r = lr[ir];
    const float margin = beta * (c - r);
    float li, dm;
    const float sg = 1.f / (1.f + expf(-margin));
    if (smoothing > 0.f) {
      li = (1.f - smoothing) * -log_sigmoid(margin) + smoothing * -log_sigmoid(-margin);
      dm = (1.f - smoothing) * (sg - 1.f) + smoothing * sg;
    } else {
      li = -log_sigmoid(margin);
      dm = sg - 1.f;
    }
    dm /= (float)P;
    v[0] += li;
    v[1] += beta * c;
    v[2] += beta * r;
    v[3] += (beta * c > beta * r) ? 1.0 : 0.0;
    v[4] += margin;
    row_coef[ic] = beta * dm;
    row_coef[ir] = -beta * dm;
  }
  block_sum<double, 5>(v, scratch);
  if (threadIdx.x == 0) {
    double rs = 0.0;
    for (int b = 0; b < B; ++b) rs += rewards ? rewards[b] : 0.0;
    const float loss = (float)(v[0] / P);
    loss_out[0] = loss;
    metrics[0] = loss;
    metrics[1] = rewards ? (float)(rs / B) : 0.f;
    metrics[2] = (float)(v[1] / P);
    metrics[3] = (float)(v[2] / P);
    metrics[4] = (float)(v[3] / P);
    metrics[5] = (float)(v[4] / P);
    metrics[6] = 0.f;
    metrics[7] = (float)P;
  }
}

// GRPO / DAPO loss kernel: 2 bulk-copy staged, 1 (default) register loads, 0 the general
// clipped-ratio kernel (IKRL_TUNE_LOSS_KERNEL; kept for A/B timing).
int lean_loss_mode() { return (int)tuning(IKRL_TUNE_LOSS_KERNEL); }

// Launch with programmatic stream serialization: the kernel may be scheduled while the previous
// kernel of the stream runs (its launch latency overlaps that kernel's tail); it calls
// griddep_wait() before touching memory.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, const char* name,
               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  IKRL_CUDA(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
  return check_launch(name);
}

// The fixed-order combine of the loss kernel's per-block partials (and its batch-level slot).
int launch_sums_reduce(const LossArgs& a, int nblocks, bool derive_token_loss, cudaStream_t s) {
  // The one-block reduce is scheduled while the loss kernel still runs and waits in-kernel for it.
  return launch_pdl(loss_sums_reduce_kernel, dim3(1), dim3(256), 0, s, "loss_sums_reduce_kernel",
                    (const double*)a.partials, nblocks, derive_token_loss ? 1 : 0, a.p.beta, a.B, a.G, a.sums);
}

int loss_grid(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(cdiv(n, 4), kLossThreads), kLossMaxBlocks)); }

}  // namespace
}  // namespace ikrl

using namespace ikrl;

extern "C" {

int ikrl_mask_count(const uint8_t* mask, int64_t n, int64_t* count_out, void* stream) {
  clear_error();
  IKRL_REQUIRE(count_out != nullptr && n >= 0 && (n == 0 || mask != nullptr), IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_mask_count: bad arguments (n=%lld)", (long long)n);
  cudaStream_t s = as_stream(stream);
  IKRL_CUDA(cudaMemsetAsync(count_out, 0, sizeof(int64_t), s));
  if (n == 0) return IKRL_OK;
  const int grid = (int)std::min<int64_t>(kNumSMs * 4, cdiv(cdiv(n, 16), 256));
  mask_count_kernel<<<std::max(grid, 1), 256, 0, s>>>(mask, n, reinterpret_cast<unsigned long long*>(count_out));
  return check_launch("mask_count_kernel");
}

int ikrl_broadcast_advantages(const float* rewards, const uint8_t* response_mask, int32_t B, int32_t T,
                              float* adv_out, void* stream) {
  clear_error();
  IKRL_REQUIRE(B >= 0 && T >= 0 && (B == 0 || (rewards && response_mask && adv_out)), IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_broadcast_advantages: bad arguments");
  if ((int64_t)B * T == 0) return IKRL_OK;
  broadcast_adv_kernel<<<B, 256, 0, as_stream(stream)>>>(rewards, response_mask, B, T, adv_out);
  return check_launch("broadcast_adv_kernel");
}

int ikrl_group_advantages(const float* rewards, const uint8_t* response_mask, const uint8_t* truncated,
                          int32_t B, int32_t T, int32_t G, int32_t filter_zero_var, float overlong_penalty,
                          float* adv_out, float* row_adv_out, void* stream) {
  clear_error();
  IKRL_REQUIRE(B >= 0 && T >= 0 && G >= 1, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_group_advantages: bad sizes B=%d T=%d G=%d", B, T, G);
  IKRL_REQUIRE(B % G == 0, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_group_advantages: B=%d is not a multiple of group_size G=%d", B, G);
  if (B == 0) return IKRL_OK;
  IKRL_REQUIRE(rewards && response_mask && adv_out, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_group_advantages: null pointer");
  return launch_pdl(group_adv_kernel, dim3(B), dim3(256), 0, as_stream(stream), "group_adv_kernel", rewards,
                    response_mask, truncated, B, T, G, filter_zero_var, overlong_penalty, adv_out, row_adv_out);
}

int ikrl_token_group_advantages(const float* token_rewards, const uint8_t* response_mask, int32_t B,
                                int32_t T, int32_t G, float* adv_out, void* stream) {
  clear_error();
  IKRL_REQUIRE(B >= 0 && T >= 0 && G >= 1 && B % G == 0, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_token_group_advantages: bad sizes B=%d T=%d G=%d", B, T, G);
  const int64_t work = (int64_t)(B / G) * T;
  if (work == 0) return IKRL_OK;
  IKRL_REQUIRE(token_rewards && response_mask && adv_out, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_token_group_advantages: null pointer");
  token_group_adv_kernel<<<(unsigned)cdiv(work, 256), 256, 0, as_stream(stream)>>>(token_rewards, response_mask,
                                                                                   B, T, G, adv_out);
  return check_launch("token_group_adv_kernel");
}

size_t ikrl_masked_moments_workspace_bytes(int64_t n) {
  (void)n;
  return 256 + (size_t)kNumSMs * 2 * 2 * sizeof(double);
}

int ikrl_masked_moments(const float* x, const uint8_t* mask, int64_t n, float* out4, void* ws, size_t ws_bytes,
                        void* stream) {
  clear_error();
  IKRL_REQUIRE(n >= 0 && out4 && (n == 0 || (x && mask)), IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_masked_moments: bad arguments");
  IKRL_REQUIRE(ws != nullptr && ws_bytes >= ikrl_masked_moments_workspace_bytes(n), IKRL_ERR_WORKSPACE,
               "ikrl_masked_moments: workspace too small (%zu < %zu)", ws_bytes,
               ikrl_masked_moments_workspace_bytes(n));
  cudaStream_t s = as_stream(stream);
  unsigned* ticket = reinterpret_cast<unsigned*>(ws);
  double* partials = reinterpret_cast<double*>(reinterpret_cast<char*>(ws) + 256);
  IKRL_CUDA(cudaMemsetAsync(ticket, 0, sizeof(unsigned), s));
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(kNumSMs * 2, cdiv(n, 256)));
  moments_pass_kernel<<<grid, 256, 0, s>>>(x, mask, n, 0, out4, partials, ticket);
  int rc = check_launch("moments_pass_kernel");
  if (rc) return rc;
  moments_pass_kernel<<<grid, 256, 0, s>>>(x, mask, n, 1, out4, partials, ticket);
  return check_launch("moments_pass_kernel");
}

int ikrl_gae_advantages(const float* rewards_b, const float* rewards_bt, const float* values,
                        const uint8_t* response_mask, int32_t B, int32_t T, float gamma, float lam,
                        float* adv_out, void* stream) {
  clear_error();
  IKRL_REQUIRE(B >= 0 && T >= 0, IKRL_ERR_INVALID_ARGUMENT, "ikrl_gae_advantages: bad sizes");
  if ((int64_t)B * T == 0) return IKRL_OK;
  IKRL_REQUIRE(values && response_mask && adv_out && (rewards_b || rewards_bt), IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_gae_advantages: null pointer");
  gae_kernel<<<B, kGaeThreads, 0, as_stream(stream)>>>(rewards_b, rewards_bt, values, response_mask, T, gamma,
                                                      lam, adv_out);
  return check_launch("gae_kernel");
}

size_t ikrl_clip_loss_workspace_bytes(int64_t n_tokens) {
  // per-block partials plus one slot for the batch-level terms
  return 256 + (size_t)(loss_grid(n_tokens) + 1) * IKRL_LOSS_NSUMS * sizeof(double);
}

int ikrl_clip_loss_fwd(const void* new_lp, int32_t lp_dtype, const float* old_lp, const float* ref_lp,
                       const float* adv, const uint8_t* mask, const float* rewards, int32_t B, int32_t T,
                       int32_t G, const int64_t* ntok,
                       const float* whiten, const float* values, const float* old_values,
                       const ikrl_loss_params* params, void* dlp_out, float* dvalues_out, double* sums_out,
                       void* ws, size_t ws_bytes, void* stream) {
  clear_error();
  const int64_t n = (int64_t)B * T;
  IKRL_REQUIRE(B >= 0 && T >= 0 && params && ntok && sums_out && (B == 0 || rewards), IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_clip_loss_fwd: bad arguments");
  IKRL_REQUIRE(G <= 0 || B % G == 0, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_clip_loss_fwd: B=%d not a multiple of group_size G=%d", B, G);
  IKRL_REQUIRE(n == 0 || (new_lp && old_lp && adv && mask), IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_clip_loss_fwd: null tensor pointer");
  IKRL_REQUIRE(lp_dtype == IKRL_DTYPE_F32 || lp_dtype == IKRL_DTYPE_BF16, IKRL_ERR_UNSUPPORTED,
               "ikrl_clip_loss_fwd: lp_dtype %d unsupported", lp_dtype);
  IKRL_REQUIRE(params->family == IKRL_LOSS_GRPO || params->family == IKRL_LOSS_PPO, IKRL_ERR_UNSUPPORTED,
               "ikrl_clip_loss_fwd: loss family %d unsupported", params->family);
  IKRL_REQUIRE((values == nullptr) == (old_values == nullptr), IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_clip_loss_fwd: values and old_values must both be given or both be NULL");
  IKRL_REQUIRE(ws != nullptr && ws_bytes >= ikrl_clip_loss_workspace_bytes(n), IKRL_ERR_WORKSPACE,
               "ikrl_clip_loss_fwd: workspace too small (%zu < %zu)", ws_bytes, ikrl_clip_loss_workspace_bytes(n));
  cudaStream_t s = as_stream(stream);
  LossArgs a;
  a.new_lp = new_lp; a.old_lp = old_lp; a.ref_lp = ref_lp; a.adv = adv; a.mask = mask; a.ntok = ntok;
  a.rewards = rewards; a.B = B; a.G = G;
  a.whiten = whiten; a.values = values; a.old_values = old_values; a.dlp = dlp_out; a.dvalues = dvalues_out;
  a.partials = reinterpret_cast<double*>(reinterpret_cast<char*>(ws) + 256);
  a.sums = sums_out; a.n = n; a.p = *params;
  const int grid = loss_grid(n);
  const bool bf = lp_dtype == IKRL_DTYPE_BF16;
  auto al = [](const void* p, uintptr_t m) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & (m - 1)) == 0; };
  const bool vec = (n % 4 == 0) && al(new_lp, bf ? 8 : 16) && al(old_lp, 16) && al(ref_lp, 16) && al(adv, 16) &&
                   al(mask, 4) && al(values, 16) && al(old_values, 16) && al(dlp_out, bf ? 8 : 16) &&
                   al(dvalues_out, 16);
  const bool has_kl = ref_lp != nullptr && params->kl_type != IKRL_KL_NONE;
  const int lean = lean_loss_mode();
  if (vec && params->family == IKRL_LOSS_GRPO && values == nullptr && whiten == nullptr && lean != 0) {
    const int kl = !has_kl ? 0 : params->kl_type == IKRL_KL_SCHULMAN ? 1 : 2;
    const bool bulk_ok = lean == 2 && n >= kBulkTile && al(new_lp, 16) && al(old_lp, 16) && al(ref_lp, 16) &&
                         al(adv, 16) && al(mask, 16);
    if (bulk_ok) {
      // one block more than tiles (block 0 takes the batch-level terms), at most two per SM
      const int bgrid = (int)std::min<int64_t>(cdiv(n, kBulkTile) + 1, (int64_t)kNumSMs * kBulkBlocksPerSM);
      const uint32_t smem = kBulkStages * (bf ? bulk_stage_bytes<true>() : bulk_stage_bytes<false>());
      int rc = 0;
#define IKRL_LAUNCH_BULK(BF, KLV)                                                                      \
  do {                                                                                                \
    IKRL_CUDA(cudaFuncSetAttribute(grpo_loss_bulk_kernel<BF, KLV>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                   (int)smem));                                                       \
    rc = launch_pdl(grpo_loss_bulk_kernel<BF, KLV>, dim3(bgrid), dim3(kBulkThreads), smem, s,          \
                    "grpo_loss_bulk_kernel", a);                                                      \
  } while (0)
      if (bf) { if (kl == 0) IKRL_LAUNCH_BULK(true, 0); else if (kl == 1) IKRL_LAUNCH_BULK(true, 1); else IKRL_LAUNCH_BULK(true, 2); }
      else { if (kl == 0) IKRL_LAUNCH_BULK(false, 0); else if (kl == 1) IKRL_LAUNCH_BULK(false, 1); else IKRL_LAUNCH_BULK(false, 2); }
#undef IKRL_LAUNCH_BULK
      return rc ? rc : launch_sums_reduce(a, token_blocks(bgrid), true, s);
    }
    int rc = 0;
#define IKRL_LAUNCH_LEAN(BF, KLV) \
  rc = launch_pdl(grpo_loss_kernel<BF, KLV>, dim3(grid), dim3(kLossThreads), 0, s, "grpo_loss_kernel", a)
    if (bf) { if (kl == 0) IKRL_LAUNCH_LEAN(true, 0); else if (kl == 1) IKRL_LAUNCH_LEAN(true, 1); else IKRL_LAUNCH_LEAN(true, 2); }
    else { if (kl == 0) IKRL_LAUNCH_LEAN(false, 0); else if (kl == 1) IKRL_LAUNCH_LEAN(false, 1); else IKRL_LAUNCH_LEAN(false, 2); }
#undef IKRL_LAUNCH_LEAN
    return rc ? rc : launch_sums_reduce(a, token_blocks(grid), true, s);
  }
  int rc = 0;
#define IKRL_LAUNCH_LOSS(FAM, BF, VEC) \
  rc = launch_pdl(clip_loss_kernel<FAM, BF, VEC>, dim3(grid), dim3(kLossThreads), 0, s, "clip_loss_kernel", a)
  if (params->family == IKRL_LOSS_GRPO) {
    if (bf) { if (vec) IKRL_LAUNCH_LOSS(IKRL_LOSS_GRPO, true, true); else IKRL_LAUNCH_LOSS(IKRL_LOSS_GRPO, true, false); }
    else { if (vec) IKRL_LAUNCH_LOSS(IKRL_LOSS_GRPO, false, true); else IKRL_LAUNCH_LOSS(IKRL_LOSS_GRPO, false, false); }
  } else {
    if (bf) { if (vec) IKRL_LAUNCH_LOSS(IKRL_LOSS_PPO, true, true); else IKRL_LAUNCH_LOSS(IKRL_LOSS_PPO, true, false); }
    else { if (vec) IKRL_LAUNCH_LOSS(IKRL_LOSS_PPO, false, true); else IKRL_LAUNCH_LOSS(IKRL_LOSS_PPO, false, false); }
  }
#undef IKRL_LAUNCH_LOSS
  return rc ? rc : launch_sums_reduce(a, token_blocks(grid), false, s);
}

int ikrl_clip_loss_finalize(const double* sums, const int64_t* ntok, const ikrl_loss_params* params,
                            float* loss_out, float* metrics_out, void* stream) {
  clear_error();
  IKRL_REQUIRE(sums && ntok && params && loss_out && metrics_out, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_clip_loss_finalize: bad arguments");
  return launch_pdl(clip_loss_finalize_kernel, dim3(1), dim3(32), 0, as_stream(stream), "clip_loss_finalize_kernel",
                    sums, ntok, *params, loss_out, metrics_out);
}

int ikrl_scale_grad(void* g, int32_t dtype, int64_t n, const float* scale, void* stream) {
  clear_error();
  IKRL_REQUIRE(n >= 0 && scale && (n == 0 || g), IKRL_ERR_INVALID_ARGUMENT, "ikrl_scale_grad: bad arguments");
  IKRL_REQUIRE(dtype == IKRL_DTYPE_F32 || dtype == IKRL_DTYPE_BF16, IKRL_ERR_UNSUPPORTED,
               "ikrl_scale_grad: dtype %d unsupported", dtype);
  if (n == 0) return IKRL_OK;
  const int grid = (int)std::min<int64_t>(kNumSMs * 8, cdiv(n, 256));
  if (dtype == IKRL_DTYPE_BF16)
    return launch_pdl(scale_grad_kernel<true>, dim3(grid), dim3(256), 0, as_stream(stream), "scale_grad_kernel", g, n,
                      scale);
  return launch_pdl(scale_grad_kernel<false>, dim3(grid), dim3(256), 0, as_stream(stream), "scale_grad_kernel", g, n,
                    scale);
}

size_t ikrl_simpo_workspace_bytes(int32_t B) { return (size_t)(B > 0 ? B : 0) * 2 * sizeof(float) + 256; }

int ikrl_simpo_fwd(const void* lp, int32_t lp_dtype, const uint8_t* mask, const float* rewards, int32_t B,
                   int32_t T, float beta, float gamma, int32_t chosen_first, float* loss_out, float* metrics_out,
                   float* row_coef_out, void* ws, size_t ws_bytes, void* stream) {
  clear_error();
  IKRL_REQUIRE(B > 0 && T >= 0 && B % 2 == 0, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_simpo_fwd: B=%d must be positive and even (chosen/rejected pairs)", B);
  IKRL_REQUIRE(lp && mask && loss_out && metrics_out && row_coef_out, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_simpo_fwd: null pointer");
  IKRL_REQUIRE(lp_dtype == IKRL_DTYPE_F32 || lp_dtype == IKRL_DTYPE_BF16, IKRL_ERR_UNSUPPORTED,
               "ikrl_simpo_fwd: lp_dtype %d unsupported", lp_dtype);
  IKRL_REQUIRE(ws && ws_bytes >= ikrl_simpo_workspace_bytes(B), IKRL_ERR_WORKSPACE,
               "ikrl_simpo_fwd: workspace too small");
  cudaStream_t s = as_stream(stream);
  float* avg = reinterpret_cast<float*>(ws);
  float* len = avg + B;
  if (lp_dtype == IKRL_DTYPE_BF16) simpo_rows_kernel<true><<<B, 256, 0, s>>>(lp, mask, T, avg, len);
  else simpo_rows_kernel<false><<<B, 256, 0, s>>>(lp, mask, T, avg, len);
  int rc = check_launch("simpo_rows_kernel");
  if (rc) return rc;
  simpo_pairs_kernel<<<1, 256, 0, s>>>(avg, len, rewards, B, beta, gamma, chosen_first, loss_out, metrics_out,
                                       row_coef_out);
  return check_launch("simpo_pairs_kernel");
}

int ikrl_simpo_bwd(const float* row_coef, const uint8_t* mask, int32_t B, int32_t T, const float* scale,
                   void* dlp_out, int32_t dlp_dtype, void* stream) {
  clear_error();
  IKRL_REQUIRE(B >= 0 && T >= 0 && scale && (B == 0 || (row_coef && mask && dlp_out)), IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_simpo_bwd: bad arguments");
  IKRL_REQUIRE(dlp_dtype == IKRL_DTYPE_F32 || dlp_dtype == IKRL_DTYPE_BF16, IKRL_ERR_UNSUPPORTED,
               "ikrl_simpo_bwd: dtype %d unsupported", dlp_dtype);
  if ((int64_t)B * T == 0) return IKRL_OK;
  if (dlp_dtype == IKRL_DTYPE_BF16) simpo_bwd_kernel<true><<<B, 256, 0, as_stream(stream)>>>(row_coef, mask, T, scale, dlp_out);
  else simpo_bwd_kernel<false><<<B, 256, 0, as_stream(stream)>>>(row_coef, mask, T, scale, dlp_out);
  return check_launch("simpo_bwd_kernel");
}

}  // extern "C"

extern "C" {

size_t ikrl_dpo_workspace_bytes(int32_t B) { return (size_t)(B > 0 ? B : 0) * sizeof(float) + 256; }

int ikrl_dpo_fwd(const void* lp, int32_t lp_dtype, const float* ref_lp, const uint8_t* mask, const float* rewards,
                 int32_t B, int32_t T, float beta, float label_smoothing, int32_t chosen_first, float* loss_out,
                 float* metrics_out, float* row_coef_out, void* ws, size_t ws_bytes, void* stream) {
  clear_error();
  IKRL_REQUIRE(B > 0 && T >= 0 && B % 2 == 0, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_dpo_fwd: B=%d must be positive and even (chosen/rejected pairs)", B);
  IKRL_REQUIRE(lp && ref_lp && mask && loss_out && metrics_out && row_coef_out, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_dpo_fwd: null pointer");
  IKRL_REQUIRE(lp_dtype == IKRL_DTYPE_F32 || lp_dtype == IKRL_DTYPE_BF16, IKRL_ERR_UNSUPPORTED,
               "ikrl_dpo_fwd: lp_dtype %d unsupported", lp_dtype);
  IKRL_REQUIRE(ws && ws_bytes >= ikrl_dpo_workspace_bytes(B), IKRL_ERR_WORKSPACE, "ikrl_dpo_fwd: workspace too small");
  cudaStream_t s = as_stream(stream);
  float* lr = reinterpret_cast<float*>(ws);
  if (lp_dtype == IKRL_DTYPE_BF16) dpo_rows_kernel<true><<<B, 256, 0, s>>>(lp, ref_lp, mask, T, lr);
  else dpo_rows_kernel<false><<<B, 256, 0, s>>>(lp, ref_lp, mask, T, lr);
  int rc = check_launch("dpo_rows_kernel");
  if (rc) return rc;
  dpo_pairs_kernel<<<1, 256, 0, s>>>(lr, rewards, B, beta, label_smoothing, chosen_first, loss_out, metrics_out,
                                     row_coef_out);
  return check_launch("dpo_pairs_kernel");
}

}  // extern "C"
