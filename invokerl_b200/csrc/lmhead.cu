// K1: fused LM-head log-prob on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces invokerl/policy.py:124-191 (`_chunked_lm_head_ce` / `_chunk_ce_fn`: F.linear then
// -F.cross_entropy, chunk by chunk under torch.utils.checkpoint) and its autograd.
//
// Forward: logits tiles S = h W^T are produced in TMEM, 128 rows x 256 vocab columns at a time,
// and consumed in place by an epilogue that keeps an online (max, sum-exp) per row and picks out
// the target logit; the [N, V] logits never reach HBM.  Partial row statistics of each vocab
// split are merged by a small combine kernel: log p = S[target] - logsumexp(S).
//
// Backward: for each chunk of rows, the same GEMM recomputes S and its epilogue writes
// dS = g * (onehot - exp(S - lse)) in bf16 to a chunk workspace; two more tcgen05 GEMMs form
// dH = dS W (A K-major, B MN-major) and dW += dS^T h (both MN-major), the latter accumulated in
// fp32.  Only one chunk of dS exists at a time.
//
// Kernel shape (one CTA per SM, 192 threads):
//   warp 0      TMA producer: 4-stage ring of {A 128x64, B 256x64} bf16 tiles, 128B swizzle
//   warp 1      TMEM allocator + MMA issuer: tcgen05.mma M=128 N=256 K=16, f32 accumulators,
//               two accumulators (2 x 256 TMEM columns) so the epilogue of tile j overlaps the
//               MMAs of tile j+1
//   warps 2-5   epilogue: tcgen05.ld, one TMEM lane (= one output row) per thread
// Every mbarrier wait is bounded (sm100::kWaitTimeoutNs); on expiry the CTA records an error,
// drains its in-flight copies and MMAs, frees TMEM and exits.
#include "common.cuh"
#include "sm100.cuh"

#include <atomic>
#include <mutex>
#include <vector>

namespace ikrl {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;
// The wide kernel runs four epilogue warps per TMEM lane quadrant, each on a quarter of the columns
// of each 256-column half of the 512-column tile (64 columns per half).
constexpr int kWideEpiWarps = 16;
constexpr int kWideGroups = kWideEpiWarps / 4;
constexpr int kWideThreads = 64 + 32 * kWideEpiWarps;
constexpr uint32_t kTileA = BM * BK * 2;  // 16 KB
constexpr uint32_t kTileB = BN * BK * 2;  // 32 KB
constexpr uint32_t kStageBytes = kTileA + kTileB;
constexpr uint32_t kSmemBytes = kStages * kStageBytes + 1024;  // + alignment slack
constexpr uint32_t kTmemCols = 2 * BN;
constexpr uint32_t kMnAtomBytes = 64 * BK * 2;  // one 64-wide MN slab of an MN-major tile: 8 KB

// EPI_LSE_CACHED: the forward's epilogue that also fills the logit cache (its own instantiation,
// so the plain forward carries none of the cache's code).
enum Epi : int { EPI_LSE = 0, EPI_DLOGITS = 1, EPI_STORE_BF16 = 2, EPI_F32 = 3, EPI_LSE_CACHED = 4 };
constexpr bool is_lse(int epi) { return epi == EPI_LSE || epi == EPI_LSE_CACHED; }
enum F32Mode : int { F32_STORE = 0, F32_ADD = 1, F32_ADD_TO_BF16 = 2 };

struct GemmParams {
  int M, N, K;            // C[M, N] = A[M, K] * B[N, K]^T
  int n_tiles;            // ceil(N / BN)
  int tiles_per_split;    // consecutive N tiles of one CTA
  int splits;             // number of N ranges (gridDim.x when split-major)
  int split_major;        // 1: blockIdx.x = split, blockIdx.y = row block; 0: the reverse
  const int64_t* ids;     // [M] target ids (LSE / DLOGITS)
  const float* lse;       // [M] (DLOGITS)
  const float* g;         // [M] upstream d loss / d logp (DLOGITS)
  float* part_m;          // [splits][M] running max, log2 units (LSE)
  float* part_s;          // [splits][M] sum of 2^(x - max) (LSE)
  float* part_t;          // [M] raw target logit, written by the split owning the target (LSE)
  uint16_t* out_bf16;     // DLOGITS: dS; STORE_BF16: output; F32 mode 2: bf16 output
  int64_t ld_bf16;
  float* out_f32;         // F32: accumulator
  int64_t ld_f32;
  int f32_mode;
  int* err;               // device error word
  int part_sets;          // LSE partial sets written (splits x column halves), set by the launcher
  int a_policy, b_policy; // L2 eviction priority of the A / B loads: 0 normal, 1 evict-last, 2 evict-first
  unsigned* lockstep;     // [npairs] tiles started per pair (zeroed per launch), or null: no pacing
  int64_t id_offset;      // first vocabulary id of W's rows (a vocab shard); 0 for the whole vocabulary
  int pace_kb, pace_lag;  // pacing: K blocks between checkpoints, checkpoints a pair may lead by
  int split_tail;         // wide kernel: how many of a tile's last K blocks run first-half-first
  int ksplits;            // wide kernel: K ranges per output tile (<= 1: one), each to its own
  int64_t ks_stride;      //   fp32 partial output, ks_stride elements apart (EPI_F32 only)
  int ds_tma;             // DLOGITS in the wide kernel: 1 = stage dS in shared memory, TMA-store it
  // Logit cache (LSE, optional): rows with slot[r] >= 0 store, per 32-column chunk, the bf16
  // numerators 2^(S log2e - m) relative to the chunk maximum m and m itself (log2 units), so the
  // backward can form dS without recomputing the logits.
  const int* slot;        // [M] cache slot of each row, -1 = not cached; null = no cache
  uint16_t* cache_q;      // [slots][ld_cache] bf16 numerators
  float* cache_m;         // [slots][n_mchunks] chunk maxima, log2 units
  int64_t ld_cache;
  int n_mchunks;
};

__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, int* err) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitTimeoutNs / 4) {
      atomicCAS(err, 0, kErrTimeoutDrain);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void st_global_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Epilogue role (warps 2..): drain accumulator tiles from TMEM, one row per thread, and apply the
// epilogue EPI.  acc_full[a] are this CTA's barriers; acc_empty[a] are the addresses the warps
// arrive on when a tile is consumed (this CTA's, or the pair leader's when cluster_arrive).
// tile_base: number of tiles this CTA consumed before this unit (accumulator ring position).
// Returns false when a wait gave up (abort).
// GROUPS: column groups; warp w drains TMEM lane quadrant w % 4 and column group (w - 2) / 4.
// SPLIT (wide tile, one accumulator): the halves complete separately (acc_full[0] when the first
// 256-column half of a tile is final, acc_full[1] for the second).  Every warp loads its columns
// of the first half into registers and releases that half (acc_empty[0]) at once, so the next
// tile's first-half MMAs start while it computes; then it does the same for the second half
// (acc_empty[1]).
// stage_smem (DLOGITS only, 0 = unused): this warp's 2 KB staging tile; the dS values of each
// 32 x 32 block are written there in the 64-byte swizzled layout of tm_store and sent to global
// memory with one TMA store per block, instead of 32 scattered row stores.
template <int EPI, int TILE_N = BN, int NBUF = 2, int GROUPS = 1, bool SPLIT = false>
__device__ __forceinline__ bool epilogue_role(const GemmParams& p, uint32_t tmem_base, int m0, int split, int t_begin,
                                              int t_end, int warp, int lane, const uint32_t (&acc_full)[2],
                                              const uint32_t (&acc_empty)[2], bool cluster_arrive,
                                              volatile int* abort_v, int tile_base = 0,
                                              const CUtensorMap* tm_store = nullptr, uint32_t stage_smem = 0,
                                              int64_t out_off = 0) {
  const int ntiles = t_end - t_begin;
  bool ok = true;
  const int q = warp & 3;  // TMEM lane quadrant this warp may access
  constexpr int kCols = TILE_N / GROUPS;  // columns of the tile this warp drains
  static_assert(!SPLIT || NBUF == 1, "split drain needs one accumulator");
  constexpr int kSegs = SPLIT ? 2 : 1;                      // column segments, drained in order
  constexpr int kSegCols = SPLIT ? TILE_N / (2 * GROUPS) : kCols;
  static_assert(!SPLIT || kSegCols % 32 == 0, "split segments are whole 32-column chunks");
  const int group = GROUPS == 1 ? 0 : (warp - 2) / 4;
  const int c_lo = group * kCols;
  const int r = q * 32 + lane;
  const int grow = m0 + r;
  const bool row_ok = grow < p.M;
  int64_t tgt = -1;
  float lse2 = 0.f, gval = 0.f;
  if constexpr (is_lse(EPI) || EPI == EPI_DLOGITS) {
    if (row_ok) tgt = p.ids[grow];
  }
  int cslot = -1;  // logit-cache slot of this row (LSE)
  bool cache_run = false;  // the warp's 32 rows have consecutive slots: one TMA store per block
  int cslot0 = 0;
  if constexpr (EPI == EPI_LSE_CACHED) {
    if (row_ok && p.slot != nullptr) cslot = p.slot[grow];
    cslot0 = __shfl_sync(0xffffffffu, cslot, 0);
    cache_run = stage_smem != 0 && __all_sync(0xffffffffu, cslot >= 0 && cslot == cslot0 + lane);
  }
  if constexpr (EPI == EPI_DLOGITS) {
    if (row_ok) {
      lse2 = p.lse[grow] * kLog2e;
      gval = p.g[grow];
      if (tgt == -100) gval = 0.f;  // ignore_index rows have zero gradient
    }
  }
  // Column index of the target in this W (a vocab shard starts at id_offset); ignore_index rows
  // keep -100, which matches no column.
  if (tgt != -100) tgt -= p.id_offset;
  float run_m = -INFINITY, run_s = 0.f, tval = 0.f;
  bool found = false;

  // The epilogue of one 32-column chunk of this thread's row, columns [col0, col0 + 32) of the
  // output (col0 < N; the chunk may end past N).  Warp-uniform control flow.
  auto chunk = [&](float* v, int col0) {
    const int nvalid = min(32, p.N - col0);
    if constexpr (is_lse(EPI)) {
      float cm = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nvalid) cm = fmaxf(cm, v[i]);
      cm *= kLog2e;
      // Target gather without a dynamically indexed register array (which would go to local
      // memory): exactly one term is v[rel] * 1, every other term adds zero.
      const int64_t rel = tgt - col0;
      if (rel >= 0 && rel < nvalid) {
        const int rr = (int)rel;
        float acc_t = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) acc_t += (i == rr) ? v[i] : 0.f;
        tval = acc_t;
        found = true;
      }
      // Numerators relative to the chunk maximum cm (in place of the logits), then the running
      // (max, sum) update; the numerators are what the logit cache stores.
      float cs = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        v[i] = i < nvalid ? fast_exp2(fmaf(v[i], kLog2e, -cm)) : 0.f;
        cs += v[i];
      }
      if (cm > run_m) {
        run_s = fmaf(run_s, fast_exp2(run_m - cm), cs);
        run_m = cm;
      } else {
        run_s = fmaf(cs, fast_exp2(cm - run_m), run_s);
      }
      if constexpr (EPI == EPI_LSE_CACHED) {
      if (cache_run) {
        // Consecutive slots: the 32 x 32 block goes out with one TMA store, as the dS blocks do.
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
        const uint32_t row_addr = stage_smem + (uint32_t)lane * 64u;
        const uint32_t sw = ((uint32_t)lane >> 1) & 3u;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          st_shared_v4(row_addr + ((((uint32_t)k) ^ sw) << 4), pack_bf16x2(v[8 * k], v[8 * k + 1]),
                       pack_bf16x2(v[8 * k + 2], v[8 * k + 3]), pack_bf16x2(v[8 * k + 4], v[8 * k + 5]),
                       pack_bf16x2(v[8 * k + 6], v[8 * k + 7]));
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tm_store, stage_smem, col0, cslot0);
          bulk_commit();
        }
      } else if (cslot >= 0) {
        uint16_t* dst = p.cache_q + (int64_t)cslot * p.ld_cache + col0;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          st_global_v4(dst + 8 * k, pack_bf16x2(v[8 * k], v[8 * k + 1]), pack_bf16x2(v[8 * k + 2], v[8 * k + 3]),
                       pack_bf16x2(v[8 * k + 4], v[8 * k + 5]), pack_bf16x2(v[8 * k + 6], v[8 * k + 7]));
      }
      if (cslot >= 0) p.cache_m[(int64_t)cslot * p.n_mchunks + (col0 >> 5)] = cm;
      }  // EPI_LSE_CACHED
    } else if constexpr (EPI == EPI_DLOGITS) {
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float p0 = fast_exp2(fmaf(v[i], kLog2e, -lse2));
        const float p1 = fast_exp2(fmaf(v[i + 1], kLog2e, -lse2));
        const float d0 = gval * (((int64_t)(col0 + i) == tgt ? 1.f : 0.f) - p0);
        const float d1 = gval * (((int64_t)(col0 + i + 1) == tgt ? 1.f : 0.f) - p1);
        w[i >> 1] = pack_bf16x2(d0, d1);
      }
      if (stage_smem != 0) {
        // One TMA store per 32 x 32 block: row `lane` goes to the staging tile with its 16-byte
        // chunks in the 64-byte swizzled order; the tensor map clips rows >= M and columns >= N.
        if (lane == 0) bulk_wait_read_all();  // the previous block's store has read the tile
        __syncwarp();
        const uint32_t row_addr = stage_smem + (uint32_t)lane * 64u;
        const uint32_t sw = ((uint32_t)lane >> 1) & 3u;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          st_shared_v4(row_addr + ((((uint32_t)k) ^ sw) << 4), w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tm_store, stage_smem, col0, m0 + q * 32);
          bulk_commit();
        }
      } else if (row_ok) {
        uint16_t* dst = p.out_bf16 + (int64_t)grow * p.ld_bf16 + col0;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (8 * k < nvalid) st_global_v4(dst + 8 * k, w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
      }
    } else if constexpr (EPI == EPI_STORE_BF16) {
      if (row_ok) {
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) w[i >> 1] = pack_bf16x2(v[i], v[i + 1]);
        uint16_t* dst = p.out_bf16 + (int64_t)grow * p.ld_bf16 + col0;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (8 * k < nvalid) st_global_v4(dst + 8 * k, w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
      }
    } else {  // EPI_F32
      if (row_ok) {
        float* dst = p.out_f32 + out_off + (int64_t)grow * p.ld_f32 + col0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (4 * k >= nvalid) break;
          float4 x = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
          if (p.f32_mode != F32_STORE) {
            const float4 o = *reinterpret_cast<const float4*>(dst + 4 * k);
            x.x += o.x; x.y += o.y; x.z += o.z; x.w += o.w;
          }
          if (p.f32_mode == F32_ADD_TO_BF16) {
            uint16_t* d16 = p.out_bf16 + (int64_t)grow * p.ld_bf16 + col0 + 4 * k;
            *reinterpret_cast<uint2*>(d16) = make_uint2(pack_bf16x2(x.x, x.y), pack_bf16x2(x.z, x.w));
          } else {
            *reinterpret_cast<float4*>(dst + 4 * k) = x;
          }
        }
      }
    }
  };

  for (int j = 0; j < ntiles; ++j) {
    const int acc = NBUF == 2 ? ((tile_base + j) & 1) : 0;
    const uint32_t acc_phase = NBUF == 2 ? ((uint32_t)((tile_base + j) >> 1) & 1u) : ((uint32_t)(tile_base + j) & 1u);
    if constexpr (EPI == EPI_F32) {
      // Pull this row's slice of the fp32 accumulator into L2 while the MMAs run, so the
      // read-modify-write below hits L2.
      if (row_ok && p.f32_mode != F32_STORE) {
#pragma unroll
        for (int sg = 0; sg < kSegs; ++sg) {
          const int n0p = (t_begin + j) * TILE_N + (SPLIT ? sg * (TILE_N / 2) + group * kSegCols : c_lo);
          const int ncols = min(kSegCols, p.N - n0p);
          if (ncols > 0)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p.out_f32 + out_off + (int64_t)grow * p.ld_f32 + n0p),
                         "r"((uint32_t)ncols * 4u)
                         : "memory");
        }
      }
    }
    if constexpr (!SPLIT) {
      if (!mbar_wait(acc_full[acc], acc_phase, abort_v, p.err, kErrTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
    }
    const int n0 = (t_begin + j) * TILE_N;
    const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * TILE_N);
    if constexpr (SPLIT) {
      // Each half has its own full barrier (the MMA issuer finishes the first half of a tile
      // before the second): wait for the half, load its columns, release it, then compute from
      // registers.
      bool waited = true;
#pragma unroll
      for (int sg = 0; sg < 2; ++sg) {
        if (!mbar_wait(acc_full[sg], acc_phase, abort_v, p.err, kErrTimeoutEpilogue)) {
          waited = false;
          break;
        }
        tc_fence_after();
        const int cs = sg * (TILE_N / 2) + group * kSegCols;
        float v[kSegCols];
#pragma unroll
        for (int cc = 0; cc < kSegCols; cc += 32) tmem_ld32p(tbase + (uint32_t)(cs + cc), v + cc);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc_empty[sg]);
#pragma unroll
        for (int cc = 0; cc < kSegCols; cc += 32)
          if (n0 + cs + cc < p.N) chunk(v + cc, n0 + cs + cc);
      }
      if (!waited) {
        ok = false;
        break;
      }
    } else {
#pragma unroll 1
      for (int c = c_lo; c < c_lo + kCols; c += 32) {
        const int col0 = n0 + c;
        if (col0 >= p.N) break;  // warp-uniform
        float v[32];
        tmem_ld32p(tbase + (uint32_t)c, v);
        tmem_wait_ld();
        chunk(v, col0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (cluster_arrive) mbar_arrive_cluster(acc_empty[acc]);
        else mbar_arrive(acc_empty[acc]);
      }
    }
  }
  if constexpr (EPI == EPI_DLOGITS || EPI == EPI_LSE_CACHED) {
    // Every TMA store of this warp has completed before the CTA can exit.
    if (stage_smem != 0 && lane == 0) bulk_wait_all();
    __syncwarp();
  }
  if constexpr (is_lse(EPI)) {
    if (row_ok && !*abort_v) {
      const int set = split * GROUPS + group;
      p.part_m[(int64_t)set * p.M + grow] = run_m;
      p.part_s[(int64_t)set * p.M + grow] = run_s;
      if (found) p.part_t[grow] = tval;
    }
  }
  return ok;
}

template <int EPI, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    lmhead_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kStages], empty_bar[kStages], acc_full[2], acc_empty[2], drain_bar;
  __shared__ uint32_t tmem_holder;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;

  const int split = p.split_major ? blockIdx.x : blockIdx.y;
  const int m_blk = p.split_major ? blockIdx.y : blockIdx.x;
  const int m0 = m_blk * BM;
  const int t_begin = split * p.tiles_per_split;
  const int t_end = min(t_begin + p.tiles_per_split, p.n_tiles);
  const int ntiles = t_end - t_begin;
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&acc_full[a]), 1);
      mbar_init(smem_u32(&acc_empty[a]), kEpiWarps);
    }
    mbar_init(smem_u32(&drain_bar), 1);
    abort_flag = 0;
    fence_barrier_init();
    fence_async_shared();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_holder;
  volatile int* abort_v = &abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && ntiles > 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued_phase[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) issued_phase[s] = -1;
      bool ok = true;
      for (int t = t_begin; t < t_end && ok; ++t) {
        const int n0 = t * BN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1u, abort_v, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full_bar[stage]);
          mbar_arrive_expect_tx(fb, kStageBytes);
          const uint32_t a_dst = smem_base + stage * kStageBytes;
          const uint32_t b_dst = a_dst + kTileA;
          const int k0 = kb * BK;
          if constexpr (!A_MN) {
            tma_load_2d(a_dst, &tmA, fb, k0, m0);
          } else {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c) tma_load_2d(a_dst + c * kMnAtomBytes, &tmA, fb, m0 + 64 * c, k0);
          }
          if constexpr (!B_MN) {
            tma_load_2d(b_dst, &tmB, fb, k0, n0);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_2d(b_dst + c * kMnAtomBytes, &tmB, fb, n0 + 64 * c, k0);
          }
          issued_phase[stage] = (int)phase;
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
      if (ok) {
        // Tail: wait until the MMA warp has released every stage, so no arrive is pending.
        for (int s = 0; s < kStages; ++s) {
          if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1u, abort_v, p.err, kErrTimeoutProducer)) break;
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      } else {
        // Abort: let every issued copy land before shared memory is released.
        for (int s = 0; s < kStages; ++s)
          if (issued_phase[s] >= 0) mbar_wait_drain(smem_u32(&full_bar[s]), (uint32_t)issued_phase[s], p.err);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && ntiles > 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int j = 0; j < ntiles && ok; ++j) {
        const int acc = j & 1;
        const uint32_t acc_phase = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(smem_u32(&acc_empty[acc]), acc_phase ^ 1u, abort_v, p.err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(smem_u32(&full_bar[stage]), phase, abort_v, p.err, kErrTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_base + stage * kStageBytes;
          const uint32_t b_addr = a_addr + kTileA;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? smem_desc(a_addr + k * 2048, kMnAtomBytes, 1024)
                                     : smem_desc(a_addr + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc(b_addr + k * 2048, kMnAtomBytes, 1024)
                                     : smem_desc(b_addr + k * 32, 16, 1024);
            mma_bf16(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          mma_commit(smem_u32(&empty_bar[stage]));
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (ok) mma_commit(smem_u32(&acc_full[acc]));
      }
      if (!ok) {
        // Abort: wait for the MMAs already issued before TMEM and shared memory go away.
        mma_commit(smem_u32(&drain_bar));
        mbar_wait_drain(smem_u32(&drain_bar), 0, p.err);
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const uint32_t af[2] = {smem_u32(&acc_full[0]), smem_u32(&acc_full[1])};
    const uint32_t ae[2] = {smem_u32(&acc_empty[0]), smem_u32(&acc_empty[1])};
    epilogue_role<EPI>(p, tmem_base, m0, split, t_begin, t_end, warp, lane, af, ae, false, abort_v);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// CTA-pair variant (cluster of two, tcgen05 cta_group::2): the pair computes a 256 x 256 tile
// per MMA; each CTA stages its own 128 A rows and 128 of the 256 B rows, so shared-memory and
// L2 traffic per MMA flop is 2/3 of the single-CTA kernel and the ring is 6 stages deep.  The
// even CTA issues the MMAs and commits to both CTAs' barriers; both CTAs run the epilogue on
// their own 128 accumulator rows and release the accumulator on the even CTA's barrier.
#ifndef IKRL_PAIR_STAGES
#define IKRL_PAIR_STAGES 6
#endif
constexpr int kPairStages = IKRL_PAIR_STAGES;
constexpr uint32_t kPairTileB = (BN / 2) * BK * 2;  // 16 KB: this CTA's half of the B tile
constexpr uint32_t kPairStageBytes = kTileA + kPairTileB;
constexpr uint32_t kPairSmemBytes = kPairStages * kPairStageBytes + 1024;

// Pacing of the persistent pairs: pairs that read the same W tiles through L2 drift apart over a
// sweep, and a tile read by a leading pair is evicted before the trailing pairs reach it.  Each
// pair publishes how many checkpoints it has passed (one per pace_kb K blocks, default 128: one per
// two tiles at K = 4096, 8 tiles at K = 1024; a long reduction such as dH over the vocabulary has
// many per tile); a pair about to pass checkpoint j waits until every unfinished pair has passed
// checkpoint j - pace_lag (default 1).  The wait is a heuristic with a short bound: after
// kPaceBoundNs without progress the pair stops pacing for the rest of the launch (a pair that is
// not resident, e.g. on a shared GPU, must not stall the others).
constexpr uint64_t kPaceBoundNs = 20000;
constexpr unsigned kPaceDone = 0xffffffffu;

__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* ptr) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_u32(unsigned* ptr, unsigned v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

// Publish "passed checkpoint j" (counted over all of this pair's units) and wait for the laggards.
__device__ __forceinline__ void pace_checkpoint(unsigned* prog, int pair_id, int npairs, int j, int lag,
                                                bool& pacing) {
  st_relaxed_u32(prog + pair_id, (unsigned)j + 1u);
  if (!pacing || j < lag) return;
  const unsigned need = (unsigned)(j + 1 - lag);
  const uint64_t t0 = globaltimer();
  while (true) {
    unsigned mn = kPaceDone;
    for (int q = 0; q < npairs; q += 8) {
      unsigned v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = (q + i < npairs) ? ld_relaxed_u32(prog + q + i) : kPaceDone;
#pragma unroll
      for (int i = 0; i < 8; ++i) mn = min(mn, v[i]);
    }
    if (mn >= need) return;
    if (globaltimer() - t0 > kPaceBoundNs) {
      pacing = false;
      return;
    }
    __nanosleep(256);
  }
}

template <int EPI, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    lmhead_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kPairStages], empty_bar[kPairStages], acc_full[2], acc_empty[2], drain_bar;
  __shared__ uint32_t tmem_holder;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t rank = cluster_ctarank();

  // Persistent pairs.  A work unit is (split, row-block pair); unit u covers split u % splits and
  // row blocks 2 * (u / splits) + {0, 1}.  Pair c processes units c, c + npairs, ...; the units
  // in flight at any time are consecutive, so pairs that run together share the B tiles of a
  // split and the A rows of a row-block pair through L2, and proceed in step.
  const int pair_id = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int m_pairs = (((p.M + BM - 1) / BM) + 1) >> 1;
  const int nunits = m_pairs * p.splits;
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&acc_full[a]), 1);
      mbar_init(smem_u32(&acc_empty[a]), 2 * kEpiWarps);
    }
    mbar_init(smem_u32(&drain_bar), 1);
    abort_flag = 0;
    fence_barrier_init();
    fence_async_shared();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(&tmem_holder), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem_base = tmem_holder;
  volatile int* abort_v = &abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool pacing = p.lockstep != nullptr && rank == 0;
      const uint64_t pol_a = l2_policy(p.a_policy);
      const uint64_t pol_b = l2_policy(p.b_policy);
      int jt = 0;
      for (int u = pair_id; u < nunits && ok; u += npairs) {
        const int split = u % p.splits;
        const int m0 = (2 * (u / p.splits) + (int)rank) * BM;
        const int t_begin = split * p.tiles_per_split;
        const int t_end = min(t_begin + p.tiles_per_split, p.n_tiles);
        for (int t = t_begin; t < t_end && ok; ++t, ++jt) {
          const int nb = t * BN + (int)rank * (BN / 2);  // this CTA's half of the N tile
          for (int kb = 0; kb < nk; ++kb) {
            const int gkb = jt * nk + kb;
            if (p.lockstep != nullptr && rank == 0 && gkb % p.pace_kb == 0)
              pace_checkpoint(p.lockstep, pair_id, npairs, gkb / p.pace_kb, p.pace_lag, pacing);
            if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1u, abort_v, p.err, kErrTimeoutProducer)) {
              ok = false;
              break;
            }
            const uint32_t fb_local = smem_u32(&full_bar[stage]);
            const uint32_t fb_leader = mapa_shared(fb_local, 0);
            if (rank == 0) mbar_arrive_expect_tx(fb_local, 2 * kPairStageBytes);
            const uint32_t a_dst = smem_base + stage * kPairStageBytes;
            const uint32_t b_dst = a_dst + kTileA;
            const int k0 = kb * BK;
            if constexpr (!A_MN) {
              tma_load_2d_pair_hint(a_dst, &tmA, fb_leader, k0, m0, pol_a);
            } else {
#pragma unroll
              for (int c = 0; c < BM / 64; ++c)
                tma_load_2d_pair_hint(a_dst + c * kMnAtomBytes, &tmA, fb_leader, m0 + 64 * c, k0, pol_a);
            }
            if constexpr (!B_MN) {
              tma_load_2d_pair_hint(b_dst, &tmB, fb_leader, k0, nb, pol_b);
            } else {
#pragma unroll
              for (int c = 0; c < BN / 128; ++c)
                tma_load_2d_pair_hint(b_dst + c * kMnAtomBytes, &tmB, fb_leader, nb + 64 * c, k0, pol_b);
            }
            if (++stage == kPairStages) { stage = 0; phase ^= 1u; }
          }
        }
      }
      if (p.lockstep != nullptr && rank == 0) st_relaxed_u32(p.lockstep + pair_id, kPaceDone);
      if (ok) {
        for (int s = 0; s < kPairStages; ++s) {
          if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1u, abort_v, p.err, kErrTimeoutProducer)) break;
          if (++stage == kPairStages) { stage = 0; phase ^= 1u; }
        }
      } else {
        // Abort: the copies' completion is counted on the even CTA's barrier, which this CTA
        // cannot wait on; give copies already issued 1 ms to land before shared memory goes away.
        for (int i = 0; i < 1000; ++i) __nanosleep(1000);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA only) ----------------
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(2 * BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int j = 0;  // tiles issued so far (accumulator ring position)
      for (int u = pair_id; u < nunits && ok; u += npairs) {
        const int split = u % p.splits;
        const int t_begin = split * p.tiles_per_split;
        const int t_end = min(t_begin + p.tiles_per_split, p.n_tiles);
        for (int t = t_begin; t < t_end && ok; ++t, ++j) {
          const int acc = j & 1;
          const uint32_t acc_phase = (uint32_t)(j >> 1) & 1u;
          if (!mbar_wait(smem_u32(&acc_empty[acc]), acc_phase ^ 1u, abort_v, p.err, kErrTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
          for (int kb = 0; kb < nk; ++kb) {
            if (!mbar_wait(smem_u32(&full_bar[stage]), phase, abort_v, p.err, kErrTimeoutMma)) { ok = false; break; }
            tc_fence_after();
            const uint32_t a_addr = smem_base + stage * kPairStageBytes;
            const uint32_t b_addr = a_addr + kTileA;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint64_t ad = A_MN ? smem_desc(a_addr + k * 2048, kMnAtomBytes, 1024)
                                       : smem_desc(a_addr + k * 32, 16, 1024);
              const uint64_t bd = B_MN ? smem_desc(b_addr + k * 2048, kMnAtomBytes, 1024)
                                       : smem_desc(b_addr + k * 32, 16, 1024);
              mma_bf16_pair(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
            }
            const uint32_t eb = smem_u32(&empty_bar[stage]);
            mma_commit_pair(mapa_shared(eb, 0));
            mma_commit_pair(mapa_shared(eb, 1));
            if (++stage == kPairStages) { stage = 0; phase ^= 1u; }
          }
          if (ok) {
            const uint32_t fb = smem_u32(&acc_full[acc]);
            mma_commit_pair(mapa_shared(fb, 0));
            mma_commit_pair(mapa_shared(fb, 1));
          }
        }
      }
      if (!ok) {
        mma_commit_pair(mapa_shared(smem_u32(&drain_bar), 0));
        mbar_wait_drain(smem_u32(&drain_bar), 0, p.err);
      }
    }
  } else {
    // ---------------- epilogue (both CTAs, own 128 rows) ----------------
    const uint32_t af[2] = {smem_u32(&acc_full[0]), smem_u32(&acc_full[1])};
    const uint32_t ae[2] = {mapa_shared(smem_u32(&acc_empty[0]), 0), mapa_shared(smem_u32(&acc_empty[1]), 0)};
    int jb = 0;
    for (int u = pair_id; u < nunits; u += npairs) {
      const int split = u % p.splits;
      const int m0 = (2 * (u / p.splits) + (int)rank) * BM;
      const int t_begin = split * p.tiles_per_split;
      const int t_end = min(t_begin + p.tiles_per_split, p.n_tiles);
      if (!epilogue_role<EPI>(p, tmem_base, m0, split, t_begin, t_end, warp, lane, af, ae, true, abort_v, jb)) break;
      jb += t_end - t_begin;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still touch its barriers or shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// Wide CTA-pair variant for long K: the pair computes a 256 x 512 tile per K step with two
// N=256 MMAs into all 512 TMEM columns.  Each CTA stages 128 A rows and 256 of the 512 B rows per
// 64-deep K block (48 KB, 4 stages), so L2 and shared-memory reads per MMA flop are 3/4 of the
// 256 x 256 pair kernel.  The single accumulator is not double-buffered; it is drained in two
// 256-column halves, and the next tile's first-half MMAs start as soon as the first half is
// drained, so only that half's drain delays the tensor pipe.
constexpr int WN = 512;
constexpr int kWideStages = 4;
constexpr uint32_t kWideTileB = (WN / 2) * BK * 2;  // 32 KB: this CTA's half of the B tile
constexpr uint32_t kWideStageBytes = kTileA + kWideTileB;
constexpr uint32_t kWideSmemBytes = kWideStages * kWideStageBytes + 1024;
// DLOGITS adds one 32 x 32 bf16 staging tile per epilogue warp for the TMA stores of dS.
constexpr uint32_t kDsStageBytes = 32 * 32 * 2;
constexpr uint32_t kWideDsSmemBytes = kWideSmemBytes + kWideEpiWarps * kDsStageBytes;
static_assert(kWideDsSmemBytes <= 232448 - 256, "wide DLOGITS kernel exceeds the shared memory of a CTA");

template <int EPI, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kWideThreads, 1)
    lmhead_gemm_wide_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kWideStages], empty_bar[kWideStages], acc_full[2], acc_empty[2], drain_bar;
  __shared__ uint32_t tmem_holder;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t rank = cluster_ctarank();
  const int pair_id = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int m_pairs = (((p.M + BM - 1) / BM) + 1) >> 1;
  const int kspl = p.ksplits > 1 ? p.ksplits : 1;
  const int nunits = m_pairs * p.splits * kspl;
  const int nk_all = (p.K + BK - 1) / BK;
  // Work unit u: K range ks (slowest, so the units in flight share it), then the row pair, then
  // the vocab split (fastest), as without K ranges.
  auto unit_of = [&](int u, int& mp, int& split, int& ks, int& kb0, int& kb1) {
    const int per = m_pairs * p.splits;
    ks = u / per;
    const int r = u - ks * per;
    split = r % p.splits;
    mp = r / p.splits;
    kb0 = (int)((int64_t)ks * nk_all / kspl);
    kb1 = (int)((int64_t)(ks + 1) * nk_all / kspl);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWideStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&acc_full[a]), 1);
      mbar_init(smem_u32(&acc_empty[a]), 2 * kWideEpiWarps);
    }
    mbar_init(smem_u32(&drain_bar), 1);
    abort_flag = 0;
    fence_barrier_init();
    fence_async_shared();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(&tmem_holder), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = tmem_holder;
  volatile int* abort_v = &abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      const uint64_t pol_a = l2_policy(p.a_policy);
      const uint64_t pol_b = l2_policy(p.b_policy);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool pacing = p.lockstep != nullptr && rank == 0;
      int gkb = 0;  // K blocks this pair has loaded
      for (int u = pair_id; u < nunits && ok; u += npairs) {
        int mp, split, ks, kb0, kb1;
        unit_of(u, mp, split, ks, kb0, kb1);
        const int m0 = (2 * mp + (int)rank) * BM;
        const int t_begin = split * p.tiles_per_split;
        const int t_end = min(t_begin + p.tiles_per_split, p.n_tiles);
        for (int t = t_begin; t < t_end && ok; ++t) {
          for (int kb = kb0; kb < kb1; ++kb, ++gkb) {
            // pacing checkpoint every pace_kb K blocks of this pair's work
            if (p.lockstep != nullptr && rank == 0 && gkb % p.pace_kb == 0)
              pace_checkpoint(p.lockstep, pair_id, npairs, gkb / p.pace_kb, p.pace_lag, pacing);
            if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1u, abort_v, p.err, kErrTimeoutProducer)) {
              ok = false;
              break;
            }
            const uint32_t fb_local = smem_u32(&full_bar[stage]);
            const uint32_t fb_leader = mapa_shared(fb_local, 0);
            if (rank == 0) mbar_arrive_expect_tx(fb_local, 2 * kWideStageBytes);
            const uint32_t a_dst = smem_base + stage * kWideStageBytes;
            const uint32_t b_dst = a_dst + kTileA;
            const int k0 = kb * BK;
            if constexpr (!A_MN) {
              tma_load_2d_pair_hint(a_dst, &tmA, fb_leader, k0, m0, pol_a);
            } else {
#pragma unroll
              for (int c = 0; c < BM / 64; ++c)
                tma_load_2d_pair_hint(a_dst + c * kMnAtomBytes, &tmA, fb_leader, m0 + 64 * c, k0, pol_a);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              // B rows of MMA h that this CTA provides: [t*512 + 256h + 128*rank, +128)
              const int nb = t * WN + h * BN + (int)rank * (BN / 2);
              const uint32_t bh = b_dst + h * ((BN / 2) * BK * 2);
              if constexpr (!B_MN) {
                tma_load_2d_pair_hint(bh, &tmB, fb_leader, k0, nb, pol_b);
              } else {
#pragma unroll
                for (int c = 0; c < BN / 128; ++c)
                  tma_load_2d_pair_hint(bh + c * kMnAtomBytes, &tmB, fb_leader, nb + 64 * c, k0, pol_b);
              }
            }
            if (++stage == kWideStages) { stage = 0; phase ^= 1u; }
          }
        }
      }
      if (p.lockstep != nullptr && rank == 0) st_relaxed_u32(p.lockstep + pair_id, kPaceDone);
      if (ok) {
        for (int s = 0; s < kWideStages; ++s) {
          if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1u, abort_v, p.err, kErrTimeoutProducer)) break;
          if (++stage == kWideStages) { stage = 0; phase ^= 1u; }
        }
      } else {
        for (int i = 0; i < 1000; ++i) __nanosleep(1000);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA only) ----------------
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(2 * BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int j = 0;
      for (int u = pair_id; u < nunits && ok; u += npairs) {
        int mp, split, ks, kb0, kb1;
        unit_of(u, mp, split, ks, kb0, kb1);
        const int nk = kb1 - kb0;  // K blocks of this unit; kb below counts from its first
        const int t_begin = split * p.tiles_per_split;
        const int t_end = min(t_begin + p.tiles_per_split, p.n_tiles);
        // MMAs of one K block into accumulator half h (TMEM columns [256h, 256h + 256)).
        auto issue_half = [&](int st, int kb, int h) {
          const uint32_t a_addr = smem_base + st * kWideStageBytes;
          const uint32_t bh = a_addr + kTileA + h * ((BN / 2) * BK * 2);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? smem_desc(a_addr + k * 2048, kMnAtomBytes, 1024)
                                     : smem_desc(a_addr + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc(bh + k * 2048, kMnAtomBytes, 1024) : smem_desc(bh + k * 32, 16, 1024);
            mma_bf16_pair(tmem_base + (uint32_t)(h * BN), ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
        };
        auto release_stage = [&](int st) {
          const uint32_t eb = smem_u32(&empty_bar[st]);
          mma_commit_pair(mapa_shared(eb, 0));
          mma_commit_pair(mapa_shared(eb, 1));
        };
        for (int t = t_begin; t < t_end && ok; ++t, ++j) {
          const uint32_t epar = ((uint32_t)j & 1u) ^ 1u;
          if (!mbar_wait(smem_u32(&acc_empty[0]), epar, abort_v, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // The first half of the accumulator is free: run its MMAs over the K blocks already
          // staged while the epilogue still drains the second half.
          const int look = min(kWideStages, nk);
          {
            int st = stage;
            uint32_t ph = phase;
            for (int kb = 0; kb < look; ++kb) {
              if (!mbar_wait(smem_u32(&full_bar[st]), ph, abort_v, p.err, kErrTimeoutMma)) { ok = false; break; }
              tc_fence_after();
              issue_half(st, kb, 0);
              if (++st == kWideStages) { st = 0; ph ^= 1u; }
            }
          }
          if (!ok) break;
          auto commit_full = [&](int h) {
            const uint32_t fb = smem_u32(&acc_full[h]);
            mma_commit_pair(mapa_shared(fb, 0));
            mma_commit_pair(mapa_shared(fb, 1));
          };
          if (look == nk) commit_full(0);  // the whole first half is issued
          if (!mbar_wait(smem_u32(&acc_empty[1]), epar, abort_v, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int kb = 0; kb < look; ++kb) {
            issue_half(stage, kb, 1);
            release_stage(stage);
            if (++stage == kWideStages) { stage = 0; phase ^= 1u; }
          }
          // The last `tail` K blocks run first-half-first: the first half is final while the
          // second half's last MMAs still run, so the epilogue drains it and releases it for the
          // next tile without idling the tensor pipe.
          const int tail = min(min(p.split_tail, kWideStages), nk - look);
          for (int kb = look; kb < nk - tail; ++kb) {
            if (!mbar_wait(smem_u32(&full_bar[stage]), phase, abort_v, p.err, kErrTimeoutMma)) { ok = false; break; }
            tc_fence_after();
            issue_half(stage, kb, 0);
            issue_half(stage, kb, 1);
            release_stage(stage);
            if (++stage == kWideStages) { stage = 0; phase ^= 1u; }
          }
          if (!ok) break;
          if (tail > 0) {
            int st = stage;
            uint32_t ph = phase;
            for (int kb = nk - tail; kb < nk; ++kb) {
              if (!mbar_wait(smem_u32(&full_bar[st]), ph, abort_v, p.err, kErrTimeoutMma)) { ok = false; break; }
              tc_fence_after();
              issue_half(st, kb, 0);
              if (++st == kWideStages) { st = 0; ph ^= 1u; }
            }
            if (!ok) break;
            commit_full(0);
            for (int kb = nk - tail; kb < nk; ++kb) {
              issue_half(stage, kb, 1);
              release_stage(stage);
              if (++stage == kWideStages) { stage = 0; phase ^= 1u; }
            }
          } else if (look < nk) {
            commit_full(0);
          }
          commit_full(1);
        }
      }
      if (!ok) {
        mma_commit_pair(mapa_shared(smem_u32(&drain_bar), 0));
        mbar_wait_drain(smem_u32(&drain_bar), 0, p.err);
      }
    }
  } else {
    // ---------------- epilogue (both CTAs, own 128 rows x 512 columns) ----------------
    const uint32_t af[2] = {smem_u32(&acc_full[0]), smem_u32(&acc_full[1])};
    const uint32_t ae[2] = {mapa_shared(smem_u32(&acc_empty[0]), 0), mapa_shared(smem_u32(&acc_empty[1]), 0)};
    const uint32_t stage = ((EPI == EPI_DLOGITS || EPI == EPI_LSE_CACHED) && p.ds_tma)
                               ? smem_base + kWideStages * kWideStageBytes + (uint32_t)(warp - 2) * kDsStageBytes
                               : 0u;
    int jb = 0;
    for (int u = pair_id; u < nunits; u += npairs) {
      int mp, split, ks, kb0, kb1;
      unit_of(u, mp, split, ks, kb0, kb1);
      const int m0 = (2 * mp + (int)rank) * BM;
      const int t_begin = split * p.tiles_per_split;
      const int t_end = min(t_begin + p.tiles_per_split, p.n_tiles);
      if (!epilogue_role<EPI, WN, 1, kWideGroups, true>(p, tmem_base, m0, split, t_begin, t_end, warp, lane, af, ae,
                                                        true, abort_v, jb, &tmC, stage, (int64_t)ks * p.ks_stride))
        break;
      jb += t_end - t_begin;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// Merge the per-split (max, sum) pairs of each row: lse = ln2 * (M + log2 sum_s s_s 2^(m_s - M)).
__global__ void lse_combine_kernel(const float* __restrict__ part_m, const float* __restrict__ part_s,
                                   const float* __restrict__ part_t, const int64_t* __restrict__ ids, int M,
                                   int V, int splits, float* __restrict__ logp, float* __restrict__ lse_out,
                                   const int* __restrict__ err) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= M) return;
  const bool bad = *err != 0;
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, part_m[(int64_t)s * M + r]);
  float sum = 0.f;
  for (int s = 0; s < splits; ++s) sum += part_s[(int64_t)s * M + r] * fast_exp2(part_m[(int64_t)s * M + r] - mx);
  const float lse = (mx + log2f(sum)) * kLn2;
  const int64_t t = ids[r];
  float lp;
  if (bad) lp = __int_as_float(0x7fc00000);
  else if (t == -100) lp = -0.f;
  else if (t < 0 || t >= V) lp = __int_as_float(0x7fc00000);
  else lp = part_t[r] - lse;
  logp[r] = lp;
  if (lse_out) lse_out[r] = bad ? __int_as_float(0x7fc00000) : lse;
}

// Vocab shard of the forward: the shard's own logsumexp and the raw target logit when the target
// id falls in this shard (-inf otherwise, so that a max over shards picks the owner's value).
__global__ void lse_shard_combine_kernel(const float* __restrict__ part_m, const float* __restrict__ part_s,
                                         const float* __restrict__ part_t, const int64_t* __restrict__ ids, int M,
                                         int64_t vocab_start, int V_shard, int splits, float* __restrict__ tlogit,
                                         float* __restrict__ lse_out, const int* __restrict__ err) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= M) return;
  const bool bad = *err != 0;
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, part_m[(int64_t)s * M + r]);
  float sum = 0.f;
  for (int s = 0; s < splits; ++s) sum += part_s[(int64_t)s * M + r] * fast_exp2(part_m[(int64_t)s * M + r] - mx);
  const float nan = __int_as_float(0x7fc00000);
  lse_out[r] = bad ? nan : (mx + log2f(sum)) * kLn2;
  const int64_t t = ids[r];
  const bool owned = t != -100 && t >= vocab_start && t < vocab_start + V_shard;
  tlogit[r] = bad ? nan : (owned ? part_t[r] : -INFINITY);
}

// log p = t - logsumexp over shards, from each shard's (target logit or -inf, shard logsumexp):
// parts[q][0][r], parts[q][1][r] for shards q < P.  Ignored rows give -0.0 and ids outside the
// vocabulary NaN, as the unsharded forward.
__global__ void vocab_parallel_combine_kernel(const float* __restrict__ parts, const int64_t* __restrict__ ids,
                                              int64_t N, int P, int64_t V_total, float* __restrict__ logp,
                                              float* __restrict__ lse_out) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= N) return;
  float mx = -INFINITY, t = -INFINITY;
  bool nan_in = false;
  for (int q = 0; q < P; ++q) {
    const float lq = parts[((int64_t)q * 2 + 1) * N + r];
    const float tq = parts[((int64_t)q * 2) * N + r];
    nan_in |= (lq != lq) || (tq != tq);
    mx = fmaxf(mx, lq);
    t = fmaxf(t, tq);
  }
  float sum = 0.f;
  for (int q = 0; q < P; ++q) sum += expf(parts[((int64_t)q * 2 + 1) * N + r] - mx);
  const float nan = __int_as_float(0x7fc00000);
  const float lse = nan_in ? nan : mx + logf(sum);
  const int64_t id = ids[r];
  float lp;
  if (id == -100) lp = -0.f;
  else if (id < 0 || id >= V_total) lp = nan;
  else lp = t - lse;
  logp[r] = lp;
  if (lse_out) lse_out[r] = lse;
}

// ---- host side ---------------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major matrix [outer, inner] with row stride `ld` elements and a
// box of {64 inner, box_outer} elements, 128-byte swizzle, zero fill out of bounds.
int make_tmap(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_outer,
              const char* what) {
  EncodeTiledFn fn = encode_fn();
  IKRL_REQUIRE(fn != nullptr, IKRL_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  IKRL_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0, IKRL_ERR_ALIGNMENT,
               "%s: base address must be 16-byte aligned", what);
  IKRL_REQUIRE((ld * 2) % 16 == 0, IKRL_ERR_ALIGNMENT, "%s: row stride %llu elements is not a multiple of 8", what,
               (unsigned long long)ld);
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {64, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  IKRL_REQUIRE(r == CUDA_SUCCESS, IKRL_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
  return IKRL_OK;
}

// Tensor map for the wide kernel's TMA stores of dS: bf16 [outer, inner] with row stride `ld`
// elements, 32 x 32 boxes (64-byte rows) in the 64-byte swizzled shared-memory layout.  Stores clip
// at the inner and outer extents.
int make_store_tmap(CUtensorMap* m, void* base, uint64_t inner, uint64_t outer, uint64_t ld, const char* what) {
  EncodeTiledFn fn = encode_fn();
  IKRL_REQUIRE(fn != nullptr, IKRL_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  IKRL_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0, IKRL_ERR_ALIGNMENT,
               "%s: base address must be 16-byte aligned", what);
  IKRL_REQUIRE((ld * 2) % 16 == 0, IKRL_ERR_ALIGNMENT, "%s: row stride %llu elements is not a multiple of 8", what,
               (unsigned long long)ld);
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {32, 32};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  IKRL_REQUIRE(r == CUDA_SUCCESS, IKRL_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
  return IKRL_OK;
}

template <int EPI, bool A_MN, bool B_MN>
int launch_gemm(const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p, int m_tiles, cudaStream_t s) {
  auto kern = lmhead_gemm_kernel<EPI, A_MN, B_MN>;
  IKRL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
  IKRL_REQUIRE(m_tiles <= 65535 || p.split_major == 0, IKRL_ERR_UNSUPPORTED, "too many row blocks (%d)", m_tiles);
  const dim3 grid = p.split_major ? dim3(p.splits, m_tiles) : dim3(m_tiles, p.splits);
  kern<<<grid, kThreads, kSmemBytes, s>>>(a, b, p);
  return check_launch("lmhead_gemm_kernel");
}

// Pair launch: a persistent 1-D grid of one CTA pair (cluster of 2) per two SMs.
// Per-pair tile counters of the pacing in the wide kernel: one array per device, zeroed before
// every launch that paces (launches on one stream are ordered; concurrent launches on other
// streams would share it, which only weakens the pacing, whose waits are bounded).
constexpr int kMaxPacedPairs = 512;
static __device__ unsigned g_pace[kMaxPacedPairs];
std::mutex g_pace_mu;
unsigned* g_pace_addr[64] = {nullptr};

int pace_array(unsigned** out) {
  int dev = 0;
  IKRL_CUDA(cudaGetDevice(&dev));
  IKRL_REQUIRE(dev >= 0 && dev < 64, IKRL_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_pace_mu);
  if (g_pace_addr[dev] == nullptr) {
    void* ptr = nullptr;
    IKRL_CUDA(cudaGetSymbolAddress(&ptr, g_pace));
    g_pace_addr[dev] = reinterpret_cast<unsigned*>(ptr);
  }
  *out = g_pace_addr[dev];
  return IKRL_OK;
}

// Pacing of the wide kernel's pairs: IKRL_TUNE_PACE is a mask over the epilogues, bit EPI set =
// launches with that epilogue are paced.  The default (-1) paces every launch except a forward
// with K < 2048: there W is a quarter of the 8B head's bytes, the forward reads little DRAM
// unpaced, and its 16-K-block tiles make the checkpoint waits a larger share.
bool pacing_enabled(int epi, int K) {
  int64_t mask = tuning(IKRL_TUNE_PACE);
  if (mask < 0) mask = K >= 2048 ? 15 : 14;
  return (mask >> (epi == EPI_LSE_CACHED ? EPI_LSE : epi)) & 1;
}
bool persistent_pairs() { return tuning(IKRL_TUNE_PERSISTENT) != 0; }

template <int EPI, bool A_MN, bool B_MN, bool WIDE>
int launch_gemm_pair(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap* c, const GemmParams& p_in,
                     int m_tiles, cudaStream_t s) {
  GemmParams p = p_in;
  auto kern = WIDE ? lmhead_gemm_wide_kernel<EPI, A_MN, B_MN> : lmhead_gemm_pair_kernel<EPI, A_MN, B_MN>;
  p.ds_tma = (WIDE && c != nullptr && (EPI == EPI_DLOGITS || EPI == EPI_LSE_CACHED)) ? 1 : 0;
  const uint32_t smem_bytes = WIDE ? (p.ds_tma ? kWideDsSmemBytes : kWideSmemBytes) : kPairSmemBytes;
  IKRL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes));
  IKRL_REQUIRE(p.split_major == 1, IKRL_ERR_UNSUPPORTED, "pair kernel needs a split-major grid");
  IKRL_REQUIRE(WIDE || p.ksplits <= 1, IKRL_ERR_UNSUPPORTED, "K ranges need the 256x512 kernel");
  IKRL_REQUIRE(p.ksplits <= 1 || (EPI == EPI_F32 && p.f32_mode == F32_STORE), IKRL_ERR_UNSUPPORTED,
               "K ranges need fp32 partial stores");
  const int64_t nunits = (int64_t)((m_tiles + 1) / 2) * p.splits * std::max(1, p.ksplits);
  IKRL_REQUIRE(nunits <= 0x3fffffffLL, IKRL_ERR_UNSUPPORTED, "too many work units (%lld)", (long long)nunits);
  int dev = 0, nsm = kNumSMs;
  IKRL_CUDA(cudaGetDevice(&dev));
  IKRL_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
  // One resident pair per two SMs; IKRL_TUNE_PERSISTENT = 0 launches one pair per unit instead.
  const bool persistent = persistent_pairs();
  const int64_t npairs = std::max<int64_t>(1, persistent ? std::min<int64_t>(nunits, nsm / 2) : nunits);
  p.lockstep = nullptr;
  p.split_tail = (int)tuning(IKRL_TUNE_SPLIT_TAIL);
  // Pacing helps the wide kernel (long tiles, W re-read across pairs); on the 256 x 256 pair
  // kernel at K = 1024 it measured 7% slower (checkpoints every 4 short tiles stall the producer).
  if (WIDE && persistent && npairs <= kMaxPacedPairs && pacing_enabled(EPI, p.K)) {
    int rc = pace_array(&p.lockstep);
    if (rc) return rc;
    IKRL_CUDA(cudaMemsetAsync(p.lockstep, 0, sizeof(unsigned) * (size_t)npairs, s));
    p.pace_kb = (int)tuning((EPI == EPI_F32 || EPI == EPI_STORE_BF16) ? IKRL_TUNE_PACE_KB_LONG : IKRL_TUNE_PACE_KB);
    p.pace_lag = (int)tuning(IKRL_TUNE_PACE_LAG);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * npairs), 1, 1);
  cfg.blockDim = dim3(WIDE ? kWideThreads : kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, b, p.ds_tma ? *c : a, p);
  if (e != cudaSuccess) {
    int nclusters = -1;
    cudaError_t e2 = cudaOccupancyMaxActiveClusters(&nclusters, kern, &cfg);
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, kern);
    (void)cudaGetLastError();
    set_error("pair kernel launch failed: %s (grid %u x %u, max active clusters %d [%s], static smem %zu, "
              "dynamic %u, max dyn %d, regs %d, max threads %d)",
              cudaGetErrorString(e), cfg.gridDim.x, cfg.gridDim.y, nclusters, cudaGetErrorString(e2), fa.sharedSizeBytes,
              smem_bytes, fa.maxDynamicSharedSizeBytes, fa.numRegs, fa.maxThreadsPerBlock);
    return IKRL_ERR_CUDA;
  }
  return check_launch("lmhead_gemm_pair_kernel");
}

// Kernel choice: CTA pairs by default; IKRL_TUNE_CTA_PAIRS = 0 (or ikrl_lmhead_set_cta_pairs(0))
// selects the single-CTA kernel.
bool use_pairs() { return tuning(IKRL_TUNE_CTA_PAIRS) != 0; }

// Wide tiles (256 x 512 per pair) for long reductions: IKRL_TUNE_WIDE 0 never, 1 always, otherwise
// when K >= 1024 (16 K blocks per tile or more; at K = 1024 the Qwen3-0.6B head ran 1.4% faster
// wide than on 256 x 256 pairs).
bool use_wide(int K) {
  const int64_t w = tuning(IKRL_TUNE_WIDE);
  if (w == 0) return false;
  if (w == 1) return true;
  return K >= 1024;
}

int64_t cdiv64(int64_t a, int64_t b);

// Busiest pair's work, in tiles, when m_pairs row pairs x ceil(n_tiles / tps) column ranges of
// tps tiles (the last range shorter) are dealt round-robin, range fastest, to npairs persistent
// pairs: the order of the pair kernels' unit loop.
int64_t pair_makespan(int64_t m_pairs, int n_tiles, int tps, int64_t npairs) {
  const int splits = (int)cdiv64(n_tiles, tps);
  const int64_t nunits = m_pairs * splits;
  const int64_t np = std::max<int64_t>(1, std::min<int64_t>(nunits, npairs));
  int64_t worst = 0;
  for (int64_t pr = 0; pr < np; ++pr) {
    int64_t tiles = 0;
    for (int64_t u = pr; u < nunits; u += np) {
      const int sp = (int)(u % splits);
      tiles += std::min(tps, n_tiles - sp * tps);
    }
    worst = std::max(worst, tiles);
  }
  return worst;
}

// Balance of the persistent pairs: the L2 rule's split count can leave a last round of units on
// a few pairs only (14 m-pairs x 11 splits = 154 units over 74 pairs runs 3 rounds where the mean
// is 2.1).  Up to 3x the hinted count, take a larger count when it shortens the busiest pair's
// work by at least 5%; more splits mean more W re-reads, so near-balanced hints stay.  Used for
// the backward's dS launches, which have no per-split workspace.  IKRL_TUNE_BALANCE_SPLITS = 0
// keeps the hint.
bool balance_splits_enabled() { return tuning(IKRL_TUNE_BALANCE_SPLITS) != 0; }

int balanced_tiles_per_split(int64_t m_tiles, int n_tiles, int splits_hint, int64_t npairs) {
  const int64_t m_pairs = (m_tiles + 1) / 2;
  int best_tps = (int)cdiv64(n_tiles, splits_hint);
  int64_t best = pair_makespan(m_pairs, n_tiles, best_tps, npairs);
  for (int sp = splits_hint + 1; sp <= std::min(3 * splits_hint, n_tiles); ++sp) {
    const int tps = (int)cdiv64(n_tiles, sp);
    if (tps == best_tps) continue;
    const int64_t ms = pair_makespan(m_pairs, n_tiles, tps, npairs);
    if (ms * 20 < best * 19) {
      best = ms;
      best_tps = tps;
    }
  }
  return best_tps;
}

// Kernel and column ranges of one K1 GEMM launch: host arithmetic only, no CUDA call.
// kind: 0 single CTAs (128 x 256), 1 CTA pairs (256 x 256), 2 wide CTA pairs (256 x 512).
// splits_hint > 0 asks for that many column ranges (fewer if the tiles run out); splits_hint <= 0
// gives every column tile its own unit.  nsm: SMs of the GPU (one persistent pair per two).
struct K1Plan {
  int kind, n_tiles, tiles_per_split, splits;
};

K1Plan plan_k1(int epi, int64_t m_tiles, int N, int K, int splits_hint, int nsm) {
  K1Plan pl{};
  pl.kind = !use_pairs() ? 0 : (use_wide(K) ? 2 : 1);
  const bool persistent = persistent_pairs();
  const int64_t npairs = std::max(1, nsm / 2);
  if (epi == EPI_STORE_BF16 && pl.kind == 2 && splits_hint <= 0 && persistent && balance_splits_enabled() &&
      tuning(IKRL_TUNE_WIDE) == -1) {
    // bf16-store launches (dH; a one-chunk bf16 dW): every column tile is a unit reducing over the
    // whole K, so a narrow N leaves few units (dH at H = 1024: 2 wide tiles per row pair; 40 row
    // pairs give 80 units, two rounds on 74 pairs where the mean is 1.08).  256-column tiles halve
    // the unit: take the 256 x 256 pair kernel when its busiest pair finishes at least 5% sooner,
    // counting its measured ~13% lower rate per flop.
    const int64_t m_pairs = (m_tiles + 1) / 2;
    const double wide_cost = 2.0 * (double)pair_makespan(m_pairs, (int)cdiv64(N, WN), 1, npairs);
    const double pair_cost = 1.13 * (double)pair_makespan(m_pairs, (int)cdiv64(N, BN), 1, npairs);
    if (pair_cost < 0.95 * wide_cost) pl.kind = 1;
  }
  pl.n_tiles = (int)cdiv64(N, pl.kind == 2 ? WN : BN);
  if (splits_hint <= 0) {
    pl.tiles_per_split = 1;
  } else {
    pl.tiles_per_split = (int)cdiv64(pl.n_tiles, splits_hint);
    if (epi == EPI_DLOGITS && pl.kind != 0 && persistent && balance_splits_enabled())
      pl.tiles_per_split = balanced_tiles_per_split(m_tiles, pl.n_tiles, splits_hint, npairs);
  }
  pl.splits = (int)cdiv64(pl.n_tiles, pl.tiles_per_split);
  return pl;
}

// A chunk's dH may be split into at most kMaxDhSplitK K ranges, whose fp32 partials take at most
// kSplitKPartElems elements (512 MB) of the backward workspace.
constexpr int kMaxDhSplitK = 16;
constexpr int64_t kSplitKPartElems = 128ll << 20;

// K ranges for a chunk's dH = dS W.  Every 256 x 512 dH tile reduces over the whole vocabulary, so
// few row tiles leave few units: the 0.6B head's 10,066 active rows are 40 row pairs x 2 column
// tiles = 80 units for 74 pairs, two rounds where the mean is 1.08.  With ks K ranges there are
// ks times the units, each storing an fp32 partial; a second kernel sums the partials in a fixed
// order.  ks minimises the busiest pair's work plus the partials' HBM write and read (in units of
// one full-vocabulary 256 x 256 tile), and is taken when that beats the undivided choice of
// plan_k1 (256 x 512, or 256 x 256 pairs) by 5%.  1 = no split.
int dh_split_k(int64_t m_tiles, int H, int V, int64_t rows, int64_t part_elems, int nsm) {
  const int64_t forced = tuning(IKRL_TUNE_DH_SPLIT_K);
  if (forced == 0 || forced == 1) return 1;
  if (!use_pairs() || !use_wide(V) || !persistent_pairs()) return 1;
  const int64_t nk = cdiv64(V, BK);
  auto fits = [&](int64_t ks) { return ks * rows * H <= part_elems && nk / ks >= 32; };
  if (forced > 1) {
    int64_t ks = std::min<int64_t>(forced, kMaxDhSplitK);
    while (ks > 1 && !fits(ks)) --ks;
    return (int)ks;
  }
  const int64_t P = std::max(1, nsm / 2);
  const int64_t m_pairs = (m_tiles + 1) / 2;
  const int64_t U = m_pairs * cdiv64(H, WN);
  if (U >= 2 * P) return 1;
  const double tile_s = 2.0 * BN * BN * (double)V / (1.4e15 / (double)P);  // one tile on one pair
  const double elem_s = 8.0 / 6.0e12;                                       // fp32 written and read
  auto cost = [&](int64_t ks) {
    return 2.0 * (double)cdiv64(U * ks, P) / (double)ks + (double)(ks * rows * H) * elem_s / tile_s;
  };
  const double undivided = std::min(2.0 * (double)cdiv64(U, P),
                                    1.13 * (double)pair_makespan(m_pairs, (int)cdiv64(H, BN), 1, P));
  int64_t best_ks = 1;
  double best = undivided;
  for (int64_t ks = 2; ks <= kMaxDhSplitK && fits(ks); ++ks) {
    const double c = cost(ks);
    if (c < best) { best = c; best_ks = ks; }
  }
  return best < 0.95 * undivided ? (int)best_ks : 1;
}

// dH rows of a split dH: out = bf16(part[0] + part[1] + ... + part[ks-1]), summed in that order.
// n4: float4 groups of one partial (rows * H / 4); the partials are n4 groups apart.
__global__ void splitk_sum_kernel(const float4* __restrict__ part, int64_t n4, int ks, uint2* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 a = part[i];
    for (int s = 1; s < ks; ++s) {
      const float4 b = part[(int64_t)s * n4 + i];
      a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    }
    out[i] = make_uint2(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w));
  }
}

// Launch one K1 GEMM with the kernel plan_k1 selects, filling in the tile ranges; p.splits holds
// the count actually used.
// c_store: tensor map of the dS chunk for the wide kernel's TMA stores (DLOGITS), or null.
template <int EPI, bool A_MN, bool B_MN>
int launch_k1(const CUtensorMap& a_single, const CUtensorMap& b_single, const CUtensorMap& a_pair,
              const CUtensorMap& b_pair, GemmParams& p, int m_tiles, int splits_hint, cudaStream_t s,
              const CUtensorMap* c_store = nullptr) {
  int dev = 0, nsm = kNumSMs;
  IKRL_CUDA(cudaGetDevice(&dev));
  IKRL_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
  const K1Plan pl = plan_k1(EPI, m_tiles, p.N, p.K, splits_hint, nsm);
  const int kind = pl.kind;
  p.n_tiles = pl.n_tiles;
  p.tiles_per_split = pl.tiles_per_split;
  p.splits = pl.splits;
  p.split_major = 1;
  p.part_sets = p.splits * (kind == 2 ? kWideGroups : 1);
  {
    // L2 policy of the A and B loads of the wide kernel (0 normal, 1 evict-last, 2 evict-first),
    // IKRL_TUNE_L2_POLICY = 10 * a + b.  Default: A (re-read by every tile of a unit) evict-last,
    // B normal; evict-first on B measured 40% more DRAM traffic.
    const int64_t pol = tuning(IKRL_TUNE_L2_POLICY);
    p.a_policy = kind == 2 ? 1 : 0;
    p.b_policy = 0;
    if (pol >= 0) {
      p.a_policy = (int)(pol / 10);
      p.b_policy = (int)(pol % 10);
    }
  }
  if (kind == 2) return launch_gemm_pair<EPI, A_MN, B_MN, true>(a_pair, b_pair, c_store, p, m_tiles, s);
  if (kind == 1) return launch_gemm_pair<EPI, A_MN, B_MN, false>(a_pair, b_pair, nullptr, p, m_tiles, s);
  return launch_gemm<EPI, A_MN, B_MN>(a_single, b_single, p, m_tiles, s);
}

int64_t cdiv64(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Vocab splits for the row-sweeping GEMMs: enough that the row blocks resident at once keep their
// A tiles in L2 (about 24 MB of hidden rows), and enough CTAs to fill the GPU.
int choose_splits(int64_t m_tiles, int n_tiles, int H) {
  // L2 share for the A rows of the units in flight.  Long reductions (the wide kernel, whose A
  // loads are marked evict-last and whose pairs are paced) keep more rows resident and split the
  // vocabulary less: at H = 4096, 40 MB gives 4 splits.
  int64_t budget_mb = H >= 2048 ? 40 : 24;
  if (tuning(IKRL_TUNE_L2_BUDGET_MB) > 0) budget_mb = tuning(IKRL_TUNE_L2_BUDGET_MB);
  const int64_t resident_rows_budget = (budget_mb << 20) / (2ll * H);   // rows whose A tiles fit the budget
  const int64_t blocks_resident = std::max<int64_t>(1, resident_rows_budget / BM);
  int64_t s = cdiv64(kNumSMs, std::min<int64_t>(blocks_resident, m_tiles));
  s = std::max<int64_t>(s, cdiv64(2 * kNumSMs, m_tiles));
  s = std::min<int64_t>(s, n_tiles);
  return (int)std::max<int64_t>(1, s);
}

struct FwdLayout {
  size_t err_off, pm_off, ps_off, pt_off, total;
  int splits, tps;
};

FwdLayout fwd_layout(int64_t N, int H, int V) {
  FwdLayout L;
  const int64_t m_tiles = cdiv64(N, BM);
  const int n_tiles = (int)cdiv64(V, BN);
  int s = choose_splits(m_tiles, n_tiles, H);
  L.tps = (int)cdiv64(n_tiles, s);
  L.splits = (int)cdiv64(n_tiles, L.tps);
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  L.err_off = 0;
  L.pm_off = 256;
  // up to kWideGroups partial sets per split (the wide kernel's column groups)
  L.ps_off = al(L.pm_off + (size_t)kWideGroups * L.splits * N * 4);
  L.pt_off = al(L.ps_off + (size_t)kWideGroups * L.splits * N * 4);
  L.total = al(L.pt_off + (size_t)N * 4);
  return L;
}

struct BwdLayout {
  size_t err_off, ds_off, dw_off, total;
  int64_t chunk, lds;
  bool need_dw32;
  // active-row compaction (rows whose upstream gradient is exactly zero are skipped)
  size_t cnt_off, nact_off, idx_off, pos_off, idc_off, lsec_off, gc_off, hc_off, part_off;
  int64_t part_elems;
  int cblocks;
};

constexpr int kCompactRows = 2048;    // rows per block of the compaction kernels
constexpr int kCompactThreads = 256;

BwdLayout bwd_layout(int64_t N, int H, int V, int64_t chunk_rows, int dweight_dtype, int accumulate) {
  BwdLayout L;
  int64_t c = chunk_rows > 0 ? chunk_rows : N;
  c = std::min<int64_t>(c, N);
  if (c < N) c = std::max<int64_t>(BM, (c / BM) * BM);
  L.chunk = std::max<int64_t>(c, 1);
  L.lds = cdiv64(V, 64) * 64;
  const int64_t nchunks = cdiv64(N, L.chunk);
  L.need_dw32 = (dweight_dtype == IKRL_DTYPE_BF16) && (nchunks > 1 || accumulate);
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  L.err_off = 0;
  L.ds_off = 256;
  L.dw_off = al(L.ds_off + (size_t)L.chunk * L.lds * 2);
  size_t o = L.dw_off + (L.need_dw32 ? al((size_t)V * H * 4) : 0);
  L.cblocks = (int)std::max<int64_t>(1, cdiv64(N, kCompactRows));
  L.cnt_off = o;   o = al(o + (size_t)2 * L.cblocks * 4);
  L.nact_off = o;  o = al(o + 16);
  L.idx_off = o;   o = al(o + (size_t)N * 4);
  L.pos_off = o;   o = al(o + (size_t)N * 4);
  L.idc_off = o;   o = al(o + (size_t)N * 8);
  L.lsec_off = o;  o = al(o + (size_t)N * 4);
  L.gc_off = o;    o = al(o + (size_t)N * 4);
  L.hc_off = o;    o = al(o + (size_t)N * H * 2);
  // fp32 partials of a dH split into K ranges (few row tiles only; see dh_split_k)
  L.part_elems = std::min<int64_t>(kSplitKPartElems, (int64_t)kMaxDhSplitK * std::min<int64_t>(N, L.chunk) * H);
  L.part_off = o;  o = al(o + (size_t)L.part_elems * 4);
  L.total = o;
  return L;
}

// ---- active-row compaction -------------------------------------------------------------------
//
// A row contributes to dHidden and dW only through g * (onehot - softmax): rows whose upstream
// gradient g is exactly zero (tokens outside the response mask) and ignore_index rows contribute
// exact zeros.  The backward gathers the other rows, in row order, into a dense block, runs the
// three GEMMs on that block only, and scatters dHidden back (zero rows elsewhere).  NaN gradients
// count as active, so they propagate as in the dense computation.

__device__ __forceinline__ bool row_active(const float* __restrict__ g, const int64_t* __restrict__ ids, int64_t r) {
  return ids[r] != -100 && g[r] != 0.f;
}

// Rows are in two classes when the forward cached logits: active rows with a cache slot (their dS
// comes from the cache) and the other active rows (their dS is recomputed by the GEMM).  The
// compaction puts the cached class first, each class in row order.  Without a cache (slot null)
// every active row is in the second class.
__device__ __forceinline__ bool row_cached(const int* __restrict__ slot, int64_t r) {
  return slot != nullptr && slot[r] >= 0;
}

// counts[b] = cached active rows of block b, counts[nb + b] = the other active rows.
__global__ void __launch_bounds__(kCompactThreads) active_count_kernel(const float* __restrict__ g,
                                                                       const int64_t* __restrict__ ids,
                                                                       const int* __restrict__ slot, int64_t N,
                                                                       int* __restrict__ counts) {
  __shared__ int wsum[2][kCompactThreads / 32];
  const int64_t r0 = (int64_t)blockIdx.x * kCompactRows;
  int cc = 0, cu = 0;
  for (int i = threadIdx.x; i < kCompactRows; i += blockDim.x) {
    const int64_t r = r0 + i;
    if (r < N && row_active(g, ids, r)) {
      if (row_cached(slot, r)) ++cc;
      else ++cu;
    }
  }
  cc = warp_sum(cc);
  cu = warp_sum(cu);
  if ((threadIdx.x & 31) == 0) {
    wsum[0][threadIdx.x >> 5] = cc;
    wsum[1][threadIdx.x >> 5] = cu;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int tc = 0, tu = 0;
    for (int w = 0; w < kCompactThreads / 32; ++w) {
      tc += wsum[0][w];
      tu += wsum[1][w];
    }
    counts[blockIdx.x] = tc;
    counts[gridDim.x + blockIdx.x] = tu;
  }
}

// Block b writes its cached active rows after those of blocks 0..b-1, and its other active rows
// after all cached rows and the other rows of blocks 0..b-1, each in row order: idx[k] = row,
// pos[row] = k (-1 for skipped rows), and the compacted ids / lse / g.  The last block writes
// n_out[0] = active rows and n_out[1] = cached active rows.
__global__ void __launch_bounds__(kCompactThreads) compact_rows_kernel(
    const float* __restrict__ g, const int64_t* __restrict__ ids, const int* __restrict__ slot,
    const float* __restrict__ lse, int64_t N, const int* __restrict__ counts, int* __restrict__ idx,
    int* __restrict__ pos, int64_t* __restrict__ ids_c, float* __restrict__ lse_c, float* __restrict__ g_c,
    int64_t* __restrict__ n_out) {
  constexpr int kWarps = kCompactThreads / 32;
  __shared__ int wt[2][kWarps];
  __shared__ int s_base[3];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nb = (int)gridDim.x;
  int pc = 0, pu = 0, tc = 0;
  for (int b = threadIdx.x; b < nb; b += blockDim.x) {
    const int c = counts[b];
    tc += c;
    if (b < (int)blockIdx.x) {
      pc += c;
      pu += counts[nb + b];
    }
  }
  pc = warp_sum(pc);
  pu = warp_sum(pu);
  tc = warp_sum(tc);
  __shared__ int red[3][kWarps];
  if (lane == 0) {
    red[0][warp] = pc;
    red[1][warp] = pu;
    red[2][warp] = tc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int a = 0, b2 = 0, c2 = 0;
    for (int w = 0; w < kWarps; ++w) {
      a += red[0][w];
      b2 += red[1][w];
      c2 += red[2][w];
    }
    s_base[0] = a;       // cached rows before this block
    s_base[1] = c2 + b2; // other rows: after every cached row and the earlier blocks' other rows
    s_base[2] = c2;      // cached rows in total
  }
  __syncthreads();
  int base_c = s_base[0], base_u = s_base[1];
  const int64_t r0 = (int64_t)blockIdx.x * kCompactRows;
  for (int off = 0; off < kCompactRows; off += kCompactThreads) {
    const int64_t r = r0 + off + threadIdx.x;
    const bool act = r < N && row_active(g, ids, r);
    const bool cached = act && row_cached(slot, r);
    const unsigned bc = __ballot_sync(0xffffffffu, cached);
    const unsigned bu = __ballot_sync(0xffffffffu, act && !cached);
    __syncthreads();  // wt is reused
    if (lane == 0) {
      wt[0][warp] = __popc(bc);
      wt[1][warp] = __popc(bu);
    }
    __syncthreads();
    int before_c = 0, before_u = 0, total_c = 0, total_u = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      before_c += (w < warp) ? wt[0][w] : 0;
      before_u += (w < warp) ? wt[1][w] : 0;
      total_c += wt[0][w];
      total_u += wt[1][w];
    }
    if (act) {
      const unsigned below = (1u << lane) - 1u;
      const int k = cached ? base_c + before_c + __popc(bc & below) : base_u + before_u + __popc(bu & below);
      idx[k] = (int)r;
      pos[r] = k;
      ids_c[k] = ids[r];
      lse_c[k] = lse[r];
      g_c[k] = g[r];
    } else if (r < N) {
      pos[r] = -1;
    }
    base_c += total_c;
    base_u += total_u;
  }
  if (blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) {
    n_out[0] = base_u;  // the last block's other rows end at the total active count
    n_out[1] = s_base[2];
  }
}

// Cache slots of the forward: rows with cache_mask[r] != 0 (all rows when null) and a target,
// numbered in row order; rows past `cap` of them get -1.  counts[b] = such rows of block b.
__device__ __forceinline__ bool row_wants_cache(const uint8_t* __restrict__ mask, const int64_t* __restrict__ ids,
                                                int64_t r) {
  return ids[r] != -100 && (mask == nullptr || mask[r] != 0);
}

__global__ void __launch_bounds__(kCompactThreads) cache_count_kernel(const uint8_t* __restrict__ mask,
                                                                      const int64_t* __restrict__ ids, int64_t N,
                                                                      int* __restrict__ counts) {
  __shared__ int wsum[kCompactThreads / 32];
  const int64_t r0 = (int64_t)blockIdx.x * kCompactRows;
  int c = 0;
  for (int i = threadIdx.x; i < kCompactRows; i += blockDim.x) {
    const int64_t r = r0 + i;
    if (r < N && row_wants_cache(mask, ids, r)) ++c;
  }
  c = warp_sum(c);
  if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < kCompactThreads / 32; ++w) t += wsum[w];
    counts[blockIdx.x] = t;
  }
}

__global__ void __launch_bounds__(kCompactThreads) cache_slot_kernel(const uint8_t* __restrict__ mask,
                                                                     const int64_t* __restrict__ ids, int64_t N,
                                                                     const int* __restrict__ counts, int64_t cap,
                                                                     int* __restrict__ slot) {
  constexpr int kWarps = kCompactThreads / 32;
  __shared__ int wtot[kWarps];
  __shared__ int s_base;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int part = 0;
  for (int b = threadIdx.x; b < (int)blockIdx.x; b += blockDim.x) part += counts[b];
  part = warp_sum(part);
  if (lane == 0) wtot[warp] = part;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < kWarps; ++w) t += wtot[w];
    s_base = t;
  }
  __syncthreads();
  int base = s_base;
  const int64_t r0 = (int64_t)blockIdx.x * kCompactRows;
  for (int off = 0; off < kCompactRows; off += kCompactThreads) {
    const int64_t r = r0 + off + threadIdx.x;
    const bool want = r < N && row_wants_cache(mask, ids, r);
    const unsigned bal = __ballot_sync(0xffffffffu, want);
    __syncthreads();
    if (lane == 0) wtot[warp] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      before += (w < warp) ? wtot[w] : 0;
      total += wtot[w];
    }
    if (r < N) {
      const int k = base + before + __popc(bal & ((1u << lane) - 1u));
      slot[r] = (want && k < cap) ? k : -1;
    }
    base += total;
  }
}

// dS of cached rows: for chunk row k (compacted row c0 + k, original row idx[c0 + k]) and column
// j < V, dS = g * ([j == t] - q * 2^(m - lse log2e)), with q the cached bf16 numerator and m its
// chunk maximum.  Block row y handles chunk rows y, y + gridDim.y, ...; a thread takes
// kDsUnroll groups of eight columns, 256 groups apart, and issues their 16-byte loads before any
// store; V must be a multiple of 8.
constexpr int kDsUnroll = 4;
__global__ void __launch_bounds__(256) ds_from_cache_kernel(
    const uint16_t* __restrict__ cache_q, const float* __restrict__ cache_m, int64_t ld_cache, int n_mchunks,
    const int* __restrict__ slot, const int* __restrict__ idx, const int64_t* __restrict__ ids_c,
    const float* __restrict__ lse_c, const float* __restrict__ g_c, int64_t c0, int64_t rows, int V,
    int64_t id_offset, uint16_t* __restrict__ ds, int64_t ld_ds) {
  const int vec = V >> 3;
  for (int64_t k = blockIdx.y; k < rows; k += gridDim.y) {
    const int64_t kc = c0 + k;
    const int64_t sl = slot[idx[kc]];
    const float lse2 = lse_c[kc] * kLog2e;
    const float gv = g_c[kc];
    const int64_t t = ids_c[kc] - id_offset;
    const uint16_t* qrow = cache_q + sl * ld_cache;
    const float* mrow = cache_m + sl * n_mchunks;
    uint16_t* drow = ds + k * ld_ds;
    for (int jb = blockIdx.x * blockDim.x * kDsUnroll + threadIdx.x; jb < vec;
         jb += gridDim.x * blockDim.x * kDsUnroll) {
      uint4 qv[kDsUnroll];
      float mv[kDsUnroll];
#pragma unroll
      for (int u = 0; u < kDsUnroll; ++u) {
        const int jv = jb + u * (int)blockDim.x;
        if (jv < vec) {
          qv[u] = *reinterpret_cast<const uint4*>(qrow + (jv << 3));
          mv[u] = mrow[jv >> 2];
        }
      }
#pragma unroll
      for (int u = 0; u < kDsUnroll; ++u) {
        const int jv = jb + u * (int)blockDim.x;
        if (jv >= vec) break;
        const int j0 = jv << 3;
        const float sc = fast_exp2(mv[u] - lse2);
        const uint32_t w[4] = {qv[u].x, qv[u].y, qv[u].z, qv[u].w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = bf16lo(w[e]) * sc, p1 = bf16hi(w[e]) * sc;
          const float d0 = gv * (((int64_t)(j0 + 2 * e) == t ? 1.f : 0.f) - p0);
          const float d1 = gv * (((int64_t)(j0 + 2 * e + 1) == t ? 1.f : 0.f) - p1);
          o[e] = pack_bf16x2(d0, d1);
        }
        *reinterpret_cast<uint4*>(drow + j0) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

// h_c[k] = h[idx[k]] for k < n, 16 bytes per thread.
__global__ void gather_rows_kernel(const uint4* __restrict__ h, const int* __restrict__ idx, int64_t n, int vec_per_row,
                                   uint4* __restrict__ h_c) {
  const int64_t total = n * vec_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = i / vec_per_row;
    const int c = (int)(i - k * vec_per_row);
    h_c[i] = h[(int64_t)idx[k] * vec_per_row + c];
  }
}

// out[r] = pos[r] >= 0 ? src[pos[r]] : 0 for every row r < N, 16 bytes per thread.
__global__ void scatter_rows_kernel(const uint4* __restrict__ src, const int* __restrict__ pos, int64_t N,
                                    int vec_per_row, uint4* __restrict__ out) {
  const int64_t total = N * vec_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec_per_row;
    const int c = (int)(i - r * vec_per_row);
    const int k = pos[r];
    out[i] = k >= 0 ? src[(int64_t)k * vec_per_row + c] : make_uint4(0u, 0u, 0u, 0u);
  }
}

// Row skipping is on unless IKRL_TUNE_SKIP_ZERO_ROWS = 0.
bool skip_zero_rows_enabled() { return tuning(IKRL_TUNE_SKIP_ZERO_ROWS) != 0; }

int check_common(const void* hidden, const void* weight, const int64_t* ids, int64_t N, int H, int V,
                 const char* what) {
  IKRL_REQUIRE(N >= 0 && H > 0 && V > 0, IKRL_ERR_INVALID_ARGUMENT, "%s: bad sizes N=%lld H=%d V=%d", what,
               (long long)N, H, V);
  IKRL_REQUIRE(H % 8 == 0, IKRL_ERR_ALIGNMENT, "%s: hidden size H=%d must be a multiple of 8 (16-byte rows)", what, H);
  IKRL_REQUIRE(N == 0 || (hidden && weight && ids), IKRL_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  IKRL_REQUIRE(N <= (int64_t)65535 * BM, IKRL_ERR_UNSUPPORTED, "%s: N=%lld rows exceeds one launch; chunk the call",
               what, (long long)N);
  return IKRL_OK;
}

}  // namespace
}  // namespace ikrl

using namespace ikrl;

// With no rows no kernel runs; the status word at the start of the workspace is still cleared so
// that ikrl_lmhead_status reads 0 after the call.
static int clear_status_word(void* ws, size_t ws_bytes, void* stream) {
  if (ws != nullptr && ws_bytes >= sizeof(int)) IKRL_CUDA(cudaMemsetAsync(ws, 0, sizeof(int), as_stream(stream)));
  return IKRL_OK;
}

// Logit cache of a forward (all null / 0: none).  mask: rows that may be cached (null = every row
// with a target); cap: cache slots; slot: [N] output, each row's slot or -1; q / m: the cache.
struct CacheArgs {
  const uint8_t* mask = nullptr;
  int64_t cap = 0;
  int* slot = nullptr;
  uint16_t* q = nullptr;
  float* m = nullptr;
};

// Workspace of the caching forward: the forward's, then the per-block counts of the slot numbering.
size_t cache_fwd_workspace_bytes(int64_t N, int H, int V) {
  const size_t base = fwd_layout(N, H, V).total;
  return base + ((((size_t)std::max<int64_t>(1, cdiv64(N, kCompactRows)) * 4) + 255) & ~size_t(255));
}

static int lmhead_fwd_impl(const char* what, const void* hidden, const void* weight, const int64_t* ids, int64_t N, int32_t H,
                    int32_t V, int64_t vocab_start, bool shard, float* logp, float* lse, void* ws, size_t ws_bytes,
                    void* stream, const CacheArgs& cache = CacheArgs()) {
  int rc = check_common(hidden, weight, ids, N, H, V, what);
  if (rc) return rc;
  if (N == 0) return clear_status_word(ws, ws_bytes, stream);
  IKRL_REQUIRE(logp != nullptr, IKRL_ERR_INVALID_ARGUMENT, "%s: output is NULL", what);
  const FwdLayout L = fwd_layout(N, H, V);
  IKRL_REQUIRE(ws != nullptr && ws_bytes >= L.total, IKRL_ERR_WORKSPACE,
               "%s: workspace %zu < %zu bytes", what, ws_bytes, L.total);
  IKRL_REQUIRE((reinterpret_cast<uintptr_t>(ws) & 255) == 0, IKRL_ERR_ALIGNMENT,
               "%s: workspace must be 256-byte aligned", what);
  cudaStream_t s = as_stream(stream);
  char* w = reinterpret_cast<char*>(ws);
  int* err = reinterpret_cast<int*>(w + L.err_off);
  IKRL_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));

  CUtensorMap ta, tb, tb2;
  if ((rc = make_tmap(&ta, hidden, H, N, H, BM, "hidden"))) return rc;
  if ((rc = make_tmap(&tb, weight, H, V, H, BN, "weight"))) return rc;
  if ((rc = make_tmap(&tb2, weight, H, V, H, BN / 2, "weight"))) return rc;
  GemmParams p{};
  p.M = (int)N; p.N = V; p.K = H;
  p.ids = ids;
  p.id_offset = vocab_start;
  p.part_m = reinterpret_cast<float*>(w + L.pm_off);
  p.part_s = reinterpret_cast<float*>(w + L.ps_off);
  p.part_t = reinterpret_cast<float*>(w + L.pt_off);
  p.err = err;
  if (cache.slot != nullptr) {
    // Number the rows that get a cache slot (row order, at most cap of them).
    int* counts = reinterpret_cast<int*>(w + L.total);
    const int nb = (int)cdiv64(N, kCompactRows);
    cache_count_kernel<<<nb, kCompactThreads, 0, s>>>(cache.mask, ids, N, counts);
    if ((rc = check_launch("cache_count_kernel"))) return rc;
    cache_slot_kernel<<<nb, kCompactThreads, 0, s>>>(cache.mask, ids, N, counts, cache.cap, cache.slot);
    if ((rc = check_launch("cache_slot_kernel"))) return rc;
    p.slot = cache.slot;
    p.cache_q = cache.q;
    p.cache_m = cache.m;
    p.ld_cache = cdiv64(V, 64) * 64;
    p.n_mchunks = (int)cdiv64(V, 32);
  }
  CUtensorMap tq;
  if (cache.slot != nullptr && cache.cap > 0)
    if ((rc = make_store_tmap(&tq, cache.q, V, cache.cap, cdiv64(V, 64) * 64, "logit cache store"))) return rc;
  const int m_tiles = (int)cdiv64(N, BM);
  if (cache.slot != nullptr && cache.cap > 0) {
    if ((rc = launch_k1<EPI_LSE_CACHED, false, false>(ta, tb, ta, tb2, p, m_tiles, L.splits, s, &tq))) return rc;
  } else {
    if ((rc = launch_k1<EPI_LSE, false, false>(ta, tb, ta, tb2, p, m_tiles, L.splits, s))) return rc;
  }
  if (shard) {
    lse_shard_combine_kernel<<<(unsigned)cdiv64(N, 256), 256, 0, s>>>(p.part_m, p.part_s, p.part_t, ids, (int)N,
                                                                      vocab_start, V, p.part_sets, logp, lse, err);
    return check_launch("lse_shard_combine_kernel");
  }
  lse_combine_kernel<<<(unsigned)cdiv64(N, 256), 256, 0, s>>>(p.part_m, p.part_s, p.part_t, ids, (int)N, V,
                                                              p.part_sets, logp, lse, err);
  return check_launch("lse_combine_kernel");
}


// cache_slot / cache_q / cache_m: the logit cache a forward filled (all null: no cache).  Active
// rows with a slot take their dS from the cache; the others are recomputed by the dS GEMM.
static int lmhead_bwd_impl(const char* what, const void* hidden, const void* weight, const int64_t* ids,
                           const float* lse, const float* dlogp, int64_t N, int32_t H, int32_t V, int64_t vocab_start,
                           int64_t chunk_rows, void* dhidden, void* dweight, int32_t dweight_dtype,
                           int32_t accumulate_dweight, void* ws, size_t ws_bytes, void* stream,
                           const int* cache_slot = nullptr, const uint16_t* cache_q = nullptr,
                           const float* cache_m = nullptr) {
  int rc = check_common(hidden, weight, ids, N, H, V, what);
  if (rc) return rc;
  IKRL_REQUIRE(dweight_dtype == IKRL_DTYPE_F32 || dweight_dtype == IKRL_DTYPE_BF16, IKRL_ERR_UNSUPPORTED,
               "%s: dweight dtype %d unsupported", what, dweight_dtype);
  IKRL_REQUIRE(!(accumulate_dweight && dweight_dtype == IKRL_DTYPE_BF16), IKRL_ERR_UNSUPPORTED,
               "%s: accumulating into a bf16 dweight is not supported; use fp32", what);
  if (N == 0) {  // no rows: dW is zero, or left as it is when accumulating
    if (dweight && !accumulate_dweight)
      IKRL_CUDA(cudaMemsetAsync(dweight, 0, (size_t)V * H * (dweight_dtype == IKRL_DTYPE_F32 ? 4 : 2),
                                as_stream(stream)));
    return clear_status_word(ws, ws_bytes, stream);
  }
  IKRL_REQUIRE(lse && dlogp && (dhidden || dweight), IKRL_ERR_INVALID_ARGUMENT,
               "%s: null pointer", what);
  const BwdLayout L = bwd_layout(N, H, V, chunk_rows, dweight_dtype, accumulate_dweight);
  IKRL_REQUIRE(ws != nullptr && ws_bytes >= L.total, IKRL_ERR_WORKSPACE,
               "%s: workspace %zu < %zu bytes", what, ws_bytes, L.total);
  IKRL_REQUIRE((reinterpret_cast<uintptr_t>(ws) & 255) == 0, IKRL_ERR_ALIGNMENT,
               "%s: workspace must be 256-byte aligned", what);
  IKRL_REQUIRE(dweight == nullptr || (reinterpret_cast<uintptr_t>(dweight) & 15) == 0, IKRL_ERR_ALIGNMENT,
               "%s: dweight must be 16-byte aligned", what);
  IKRL_REQUIRE(dhidden == nullptr || (reinterpret_cast<uintptr_t>(dhidden) & 15) == 0, IKRL_ERR_ALIGNMENT,
               "%s: dhidden must be 16-byte aligned", what);
  cudaStream_t s = as_stream(stream);
  char* w = reinterpret_cast<char*>(ws);
  int* err = reinterpret_cast<int*>(w + L.err_off);
  uint16_t* dS = reinterpret_cast<uint16_t*>(w + L.ds_off);
  float* dw32 = L.need_dw32 ? reinterpret_cast<float*>(w + L.dw_off) : nullptr;
  IKRL_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
  const int n_vt = (int)cdiv64(V, BN);
  int nsm = kNumSMs;
  {
    int dev = 0;
    IKRL_CUDA(cudaGetDevice(&dev));
    IKRL_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
  }

  // Rows the GEMMs run on: all N, or the compacted active rows.
  const uint16_t* hsrc = reinterpret_cast<const uint16_t*>(hidden);
  const int64_t* idsrc = ids;
  const float* lsesrc = lse;
  const float* gsrc = dlogp;
  int64_t Nw = N;
  uint16_t* dh_out = reinterpret_cast<uint16_t*>(dhidden);  // where the dH GEMMs write
  const int* pos = nullptr;                                  // set when dH must be scattered back
  const int* idx_c = nullptr;                                // compacted row -> row
  int64_t n_cached = 0;                                      // leading compacted rows whose dS is cached
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  IKRL_CUDA(cudaStreamIsCapturing(s, &cap));
  if (skip_zero_rows_enabled() && cap == cudaStreamCaptureStatusNone && N <= INT32_MAX) {
    int* counts = reinterpret_cast<int*>(w + L.cnt_off);
    int64_t* n_act_d = reinterpret_cast<int64_t*>(w + L.nact_off);
    int* idx = reinterpret_cast<int*>(w + L.idx_off);
    int* posw = reinterpret_cast<int*>(w + L.pos_off);
    int64_t* ids_c = reinterpret_cast<int64_t*>(w + L.idc_off);
    float* lse_c = reinterpret_cast<float*>(w + L.lsec_off);
    float* g_c = reinterpret_cast<float*>(w + L.gc_off);
    uint16_t* h_c = reinterpret_cast<uint16_t*>(w + L.hc_off);
    const int nb = (int)cdiv64(N, kCompactRows);
    active_count_kernel<<<nb, kCompactThreads, 0, s>>>(dlogp, ids, cache_slot, N, counts);
    if ((rc = check_launch("active_count_kernel"))) return rc;
    compact_rows_kernel<<<nb, kCompactThreads, 0, s>>>(dlogp, ids, cache_slot, lse, N, counts, idx, posw, ids_c,
                                                        lse_c, g_c, n_act_d);
    if ((rc = check_launch("compact_rows_kernel"))) return rc;
    // The chunk plan depends on the active counts: read them back (one stream synchronisation).
    int64_t counts_h[2] = {0, 0};
    IKRL_CUDA(cudaMemcpyAsync(counts_h, n_act_d, 2 * sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    IKRL_CUDA(cudaStreamSynchronize(s));
    const int64_t n_act = counts_h[0];
    n_cached = counts_h[1];
    IKRL_REQUIRE(n_act >= 0 && n_act <= N && n_cached >= 0 && n_cached <= n_act, IKRL_ERR_DEVICE,
                 "%s: bad active-row counts %lld, %lld", what, (long long)n_act, (long long)n_cached);
    if (n_act == 0) {
      if (dhidden) IKRL_CUDA(cudaMemsetAsync(dhidden, 0, (size_t)N * H * 2, s));
      if (dweight && !accumulate_dweight)
        IKRL_CUDA(cudaMemsetAsync(dweight, 0, (size_t)V * H * (dweight_dtype == IKRL_DTYPE_F32 ? 4 : 2), s));
      return IKRL_OK;
    }
    if (n_act < N || n_cached > 0) {  // cached rows come first, so the order differs from the rows'
      const int vpr = H / 8;
      const int gb = (int)std::min<int64_t>(cdiv64(n_act * vpr, 256), 148ll * 16);
      gather_rows_kernel<<<gb, 256, 0, s>>>(reinterpret_cast<const uint4*>(hidden), idx, n_act, vpr,
                                            reinterpret_cast<uint4*>(h_c));
      if ((rc = check_launch("gather_rows_kernel"))) return rc;
      hsrc = h_c; idsrc = ids_c; lsesrc = lse_c; gsrc = g_c; Nw = n_act; idx_c = idx;
      // dH of a chunk overwrites that chunk's gathered rows once dW has read them.
      if (dhidden) { dh_out = h_c; pos = posw; }
    }
  }

  const BwdLayout Lw = bwd_layout(Nw, H, V, chunk_rows, dweight_dtype, accumulate_dweight);
  const int64_t chunk = std::min(L.chunk, Lw.chunk);
  // Chunks: first the cached rows [0, n_cached), then the others, so every chunk takes its dS one
  // way (from the cache, or by the recompute GEMM).
  struct Chunk {
    int64_t c0, rows;
    bool cached;
  };
  std::vector<Chunk> chunks;
  for (int seg = 0; seg < 2; ++seg) {
    const int64_t a0 = seg == 0 ? 0 : n_cached, a1 = seg == 0 ? n_cached : Nw;
    for (int64_t c0 = a0; c0 < a1; c0 += chunk) chunks.push_back({c0, std::min<int64_t>(chunk, a1 - c0), seg == 0});
  }
  const int64_t nchunks = (int64_t)chunks.size();
  const bool use_dw32 = (dweight_dtype == IKRL_DTYPE_BF16) && nchunks > 1;

  CUtensorMap t_w_k, t_w_k2, t_w_mn;
  if ((rc = make_tmap(&t_w_k, weight, H, V, H, BN, "weight"))) return rc;
  if ((rc = make_tmap(&t_w_k2, weight, H, V, H, BN / 2, "weight"))) return rc;
  if ((rc = make_tmap(&t_w_mn, weight, H, V, H, 64, "weight^T"))) return rc;

  for (int64_t ci = 0; ci < nchunks; ++ci) {
    const int64_t c0 = chunks[ci].c0;
    const int64_t rows = chunks[ci].rows;
    const int m_tiles = (int)cdiv64(rows, BM);
    const uint16_t* hc = hsrc + c0 * H;
    // 1) dS = g * (onehot - softmax(h W^T)) for this chunk: from the logit cache, or recomputed
    if (chunks[ci].cached) {
      const dim3 grid((unsigned)std::max<int64_t>(1, cdiv64(V / 8, 256 * kDsUnroll)),
                      (unsigned)std::min<int64_t>(rows, 65535));
      ds_from_cache_kernel<<<grid, 256, 0, s>>>(cache_q, cache_m, L.lds, (int)cdiv64(V, 32), cache_slot, idx_c,
                                                idsrc, lsesrc, gsrc, c0, rows, V, vocab_start, dS, L.lds);
      if ((rc = check_launch("ds_from_cache_kernel"))) return rc;
    } else {
      CUtensorMap ta, tds;
      if ((rc = make_tmap(&ta, hc, H, rows, H, BM, "hidden chunk"))) return rc;
      if ((rc = make_store_tmap(&tds, dS, V, rows, L.lds, "dS store"))) return rc;
      GemmParams p{};
      p.M = (int)rows; p.N = V; p.K = H;
      const int sp = choose_splits(m_tiles, n_vt, H);
      p.ids = idsrc + c0; p.lse = lsesrc + c0; p.g = gsrc + c0;
      p.id_offset = vocab_start;
      p.out_bf16 = dS; p.ld_bf16 = L.lds;
      p.err = err;
      if ((rc = launch_k1<EPI_DLOGITS, false, false>(ta, t_w_k, ta, t_w_k2, p, m_tiles, sp, s, &tds))) return rc;
    }
    // 2) dW (+)= dS^T h[chunk]
    if (dweight) {
      CUtensorMap ta, tb;
      if ((rc = make_tmap(&ta, dS, V, rows, L.lds, 64, "dS^T"))) return rc;
      if ((rc = make_tmap(&tb, hc, H, rows, H, 64, "hidden chunk^T"))) return rc;
      GemmParams p{};
      p.M = V; p.N = H; p.K = (int)rows;
      p.err = err;
      const int v_tiles = (int)cdiv64(V, BM);
      const bool last = ci == nchunks - 1;
      if (dweight_dtype == IKRL_DTYPE_BF16 && !use_dw32) {
        p.out_bf16 = reinterpret_cast<uint16_t*>(dweight); p.ld_bf16 = H;
        if ((rc = launch_k1<EPI_STORE_BF16, true, true>(ta, tb, ta, tb, p, v_tiles, 0, s))) return rc;
      } else {
        if (dweight_dtype == IKRL_DTYPE_F32) {
          p.out_f32 = reinterpret_cast<float*>(dweight);
          p.f32_mode = (ci == 0 && !accumulate_dweight) ? F32_STORE : F32_ADD;
        } else {
          p.out_f32 = dw32;
          p.out_bf16 = reinterpret_cast<uint16_t*>(dweight); p.ld_bf16 = H;
          p.f32_mode = last ? F32_ADD_TO_BF16 : (ci == 0 ? F32_STORE : F32_ADD);
        }
        p.ld_f32 = H;
        if ((rc = launch_k1<EPI_F32, true, true>(ta, tb, ta, tb, p, v_tiles, 0, s))) return rc;
      }
    }
    // 3) dH[chunk] = dS W, whole or as K-range partials summed afterwards
    if (dhidden) {
      CUtensorMap ta;
      if ((rc = make_tmap(&ta, dS, V, rows, L.lds, BM, "dS"))) return rc;
      GemmParams p{};
      p.M = (int)rows; p.N = H; p.K = V;
      p.err = err;
      const int ks = dh_split_k(m_tiles, H, V, rows, L.part_elems, nsm);
      if (ks > 1) {
        float* part = reinterpret_cast<float*>(w + L.part_off);
        p.out_f32 = part; p.ld_f32 = H; p.f32_mode = F32_STORE;
        p.ksplits = ks; p.ks_stride = rows * H;
        if ((rc = launch_k1<EPI_F32, false, true>(ta, t_w_mn, ta, t_w_mn, p, m_tiles, 0, s))) return rc;
        const int64_t n4 = rows * H / 4;
        const int gb = (int)std::min<int64_t>(cdiv64(n4, 256), 148ll * 8);
        splitk_sum_kernel<<<gb, 256, 0, s>>>(reinterpret_cast<const float4*>(part), n4, ks,
                                             reinterpret_cast<uint2*>(dh_out + c0 * H));
        if ((rc = check_launch("splitk_sum_kernel"))) return rc;
      } else {
        p.out_bf16 = dh_out + c0 * H; p.ld_bf16 = H;
        if ((rc = launch_k1<EPI_STORE_BF16, false, true>(ta, t_w_mn, ta, t_w_mn, p, m_tiles, 0, s))) return rc;
      }
    }
  }
  if (pos != nullptr) {
    const int vpr = H / 8;
    const int gb = (int)std::min<int64_t>(cdiv64(N * vpr, 256), 148ll * 16);
    scatter_rows_kernel<<<gb, 256, 0, s>>>(reinterpret_cast<const uint4*>(dh_out), pos, N, vpr,
                                           reinterpret_cast<uint4*>(dhidden));
    if ((rc = check_launch("scatter_rows_kernel"))) return rc;
  }
  return IKRL_OK;
}


extern "C" {

size_t ikrl_lmhead_fwd_workspace_bytes(int64_t N, int32_t H, int32_t V) {
  if (N <= 0 || H <= 0 || V <= 0) return 256;
  return fwd_layout(N, H, V).total;
}

int ikrl_lmhead_logprob_fwd(const void* hidden, const void* weight, const int64_t* ids, int64_t N, int32_t H,
                            int32_t V, float* logp, float* lse, void* ws, size_t ws_bytes, void* stream) {
  clear_error();
  return lmhead_fwd_impl("ikrl_lmhead_logprob_fwd", hidden, weight, ids, N, H, V, 0, false, logp, lse, ws, ws_bytes,
                         stream);
}

int ikrl_lmhead_shard_fwd(const void* hidden, const void* weight_shard, const int64_t* ids, int64_t N, int32_t H,
                          int32_t V_shard, int64_t vocab_start, float* tlogit, float* lse_shard, void* ws,
                          size_t ws_bytes, void* stream) {
  clear_error();
  IKRL_REQUIRE(vocab_start >= 0, IKRL_ERR_INVALID_ARGUMENT, "ikrl_lmhead_shard_fwd: vocab_start %lld < 0",
               (long long)vocab_start);
  IKRL_REQUIRE(N == 0 || lse_shard != nullptr, IKRL_ERR_INVALID_ARGUMENT, "ikrl_lmhead_shard_fwd: lse_shard is NULL");
  return lmhead_fwd_impl("ikrl_lmhead_shard_fwd", hidden, weight_shard, ids, N, H, V_shard, vocab_start, true, tlogit,
                         lse_shard, ws, ws_bytes, stream);
}

int ikrl_vocab_parallel_combine(const float* parts, const int64_t* ids, int64_t N, int32_t P, int64_t V_total,
                                float* logp, float* lse, void* stream) {
  clear_error();
  IKRL_REQUIRE(N >= 0 && P >= 1 && V_total > 0, IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_vocab_parallel_combine: bad sizes N=%lld P=%d V=%lld", (long long)N, P, (long long)V_total);
  if (N == 0) return IKRL_OK;
  IKRL_REQUIRE(parts && ids && logp, IKRL_ERR_INVALID_ARGUMENT, "ikrl_vocab_parallel_combine: null pointer");
  vocab_parallel_combine_kernel<<<(unsigned)cdiv64(N, 256), 256, 0, as_stream(stream)>>>(parts, ids, N, P, V_total,
                                                                                        logp, lse);
  return check_launch("vocab_parallel_combine_kernel");
}

size_t ikrl_lmhead_bwd_workspace_bytes(int64_t N, int32_t H, int32_t V, int64_t chunk_rows, int32_t dweight_dtype,
                                       int32_t accumulate_dweight) {
  if (N <= 0 || H <= 0 || V <= 0) return 256;
  return bwd_layout(N, H, V, chunk_rows, dweight_dtype, accumulate_dweight).total;
}

int ikrl_lmhead_logprob_bwd(const void* hidden, const void* weight, const int64_t* ids, const float* lse,
                            const float* dlogp, int64_t N, int32_t H, int32_t V, int64_t chunk_rows, void* dhidden,
                            void* dweight, int32_t dweight_dtype, int32_t accumulate_dweight, void* ws,
                            size_t ws_bytes, void* stream) {
  clear_error();
  return lmhead_bwd_impl("ikrl_lmhead_logprob_bwd", hidden, weight, ids, lse, dlogp, N, H, V, 0, chunk_rows, dhidden,
                         dweight, dweight_dtype, accumulate_dweight, ws, ws_bytes, stream);
}

int ikrl_lmhead_cache_row_elems(int32_t V, int64_t* q_elems, int64_t* m_elems) {
  clear_error();
  IKRL_REQUIRE(V > 0 && q_elems && m_elems, IKRL_ERR_INVALID_ARGUMENT, "ikrl_lmhead_cache_row_elems: bad arguments");
  *q_elems = cdiv64(V, 64) * 64;
  *m_elems = cdiv64(V, 32);
  return IKRL_OK;
}

size_t ikrl_lmhead_cache_fwd_workspace_bytes(int64_t N, int32_t H, int32_t V) {
  if (N <= 0 || H <= 0 || V <= 0) return 256;
  return cache_fwd_workspace_bytes(N, H, V);
}

int ikrl_lmhead_logprob_fwd_cached(const void* hidden, const void* weight, const int64_t* ids, int64_t N, int32_t H,
                                   int32_t V, float* logp, float* lse, const uint8_t* cache_mask, int64_t cache_rows,
                                   int32_t* cache_slot, void* cache_q, float* cache_m, void* ws, size_t ws_bytes,
                                   void* stream) {
  clear_error();
  const char* what = "ikrl_lmhead_logprob_fwd_cached";
  IKRL_REQUIRE(V % 8 == 0, IKRL_ERR_UNSUPPORTED, "%s: the logit cache needs V (%d) to be a multiple of 8", what, V);
  IKRL_REQUIRE(cache_rows >= 0, IKRL_ERR_INVALID_ARGUMENT, "%s: cache_rows %lld < 0", what, (long long)cache_rows);
  IKRL_REQUIRE(N == 0 || (cache_slot && lse && (cache_rows == 0 || (cache_q && cache_m))), IKRL_ERR_INVALID_ARGUMENT,
               "%s: null pointer", what);
  IKRL_REQUIRE((reinterpret_cast<uintptr_t>(cache_q) & 15) == 0 && (reinterpret_cast<uintptr_t>(cache_m) & 3) == 0,
               IKRL_ERR_ALIGNMENT, "%s: cache_q must be 16-byte and cache_m 4-byte aligned", what);
  const size_t need = N > 0 ? cache_fwd_workspace_bytes(N, H, V) : 0;
  IKRL_REQUIRE(N == 0 || (ws != nullptr && ws_bytes >= need), IKRL_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes",
               what, ws_bytes, need);
  CacheArgs c;
  c.mask = cache_mask;
  c.cap = cache_rows;
  c.slot = cache_slot;
  c.q = reinterpret_cast<uint16_t*>(cache_q);
  c.m = cache_m;
  return lmhead_fwd_impl(what, hidden, weight, ids, N, H, V, 0, false, logp, lse, ws, ws_bytes, stream, c);
}

int ikrl_lmhead_logprob_bwd_cached(const void* hidden, const void* weight, const int64_t* ids, const float* lse,
                                   const float* dlogp, int64_t N, int32_t H, int32_t V, int64_t chunk_rows,
                                   void* dhidden, void* dweight, int32_t dweight_dtype, int32_t accumulate_dweight,
                                   const int32_t* cache_slot, const void* cache_q, const float* cache_m, void* ws,
                                   size_t ws_bytes, void* stream) {
  clear_error();
  IKRL_REQUIRE(V % 8 == 0, IKRL_ERR_UNSUPPORTED, "ikrl_lmhead_logprob_bwd_cached: the logit cache needs V (%d) to "
               "be a multiple of 8", V);
  IKRL_REQUIRE(N == 0 || (cache_slot && cache_q && cache_m), IKRL_ERR_INVALID_ARGUMENT,
               "ikrl_lmhead_logprob_bwd_cached: null cache pointer");
  return lmhead_bwd_impl("ikrl_lmhead_logprob_bwd_cached", hidden, weight, ids, lse, dlogp, N, H, V, 0, chunk_rows,
                         dhidden, dweight, dweight_dtype, accumulate_dweight, ws, ws_bytes, stream, cache_slot,
                         reinterpret_cast<const uint16_t*>(cache_q), cache_m);
}

int ikrl_lmhead_shard_bwd(const void* hidden, const void* weight_shard, const int64_t* ids, const float* lse,
                          const float* dlogp, int64_t N, int32_t H, int32_t V_shard, int64_t vocab_start,
                          int64_t chunk_rows, void* dhidden_partial, void* dweight_shard, int32_t dweight_dtype,
                          int32_t accumulate_dweight, void* ws, size_t ws_bytes, void* stream) {
  clear_error();
  IKRL_REQUIRE(vocab_start >= 0, IKRL_ERR_INVALID_ARGUMENT, "ikrl_lmhead_shard_bwd: vocab_start %lld < 0",
               (long long)vocab_start);
  return lmhead_bwd_impl("ikrl_lmhead_shard_bwd", hidden, weight_shard, ids, lse, dlogp, N, H, V_shard, vocab_start,
                         chunk_rows, dhidden_partial, dweight_shard, dweight_dtype, accumulate_dweight, ws, ws_bytes,
                         stream);
}

int ikrl_lmhead_set_cta_pairs(int32_t enable) {
  int64_t prev = 1;
  ikrl_set_tuning(IKRL_TUNE_CTA_PAIRS, enable ? 1 : 0, &prev);
  return (int)prev;
}

int ikrl_lmhead_plan(int32_t gemm, int64_t rows, int32_t H, int32_t V, int32_t num_sms, int32_t* plan_out) {
  clear_error();
  IKRL_REQUIRE(gemm >= 0 && gemm <= 4, IKRL_ERR_INVALID_ARGUMENT, "ikrl_lmhead_plan: gemm %d not in 0..4", gemm);
  IKRL_REQUIRE(rows > 0 && rows <= (int64_t)65535 * BM && H > 0 && V > 0 && num_sms >= 2 && plan_out,
               IKRL_ERR_INVALID_ARGUMENT, "ikrl_lmhead_plan: bad arguments");
  const int64_t row_tiles = cdiv64(rows, BM);
  K1Plan pl{};
  if (gemm == 0)  // forward: the hint is the workspace's split count
    pl = plan_k1(EPI_LSE, row_tiles, V, H, fwd_layout(rows, H, V).splits, num_sms);
  else if (gemm == 1)  // dS recompute of one backward chunk of `rows` rows
    pl = plan_k1(EPI_DLOGITS, row_tiles, V, H, choose_splits(row_tiles, (int)cdiv64(V, BN), H), num_sms);
  else if (gemm == 2)  // dW += dS^T h over the chunk, fp32 accumulator
    pl = plan_k1(EPI_F32, cdiv64(V, BM), H, (int)rows, 0, num_sms);
  else if (gemm == 3)  // dH = dS W of the chunk, undivided
    pl = plan_k1(EPI_STORE_BF16, row_tiles, H, V, 0, num_sms);
  if (gemm == 4) {  // K ranges of that dH (1 = undivided), with the partial buffer of such a chunk
    const int64_t part = std::min<int64_t>(kSplitKPartElems, (int64_t)kMaxDhSplitK * rows * H);
    plan_out[0] = dh_split_k(row_tiles, H, V, rows, part, num_sms);
    plan_out[1] = plan_out[2] = plan_out[3] = 0;
    return IKRL_OK;
  }
  plan_out[0] = pl.kind;
  plan_out[1] = pl.n_tiles;
  plan_out[2] = pl.tiles_per_split;
  plan_out[3] = pl.splits;
  return IKRL_OK;
}

int ikrl_lmhead_status(const void* ws, int32_t* status_out, void* stream) {
  clear_error();
  IKRL_REQUIRE(ws && status_out, IKRL_ERR_INVALID_ARGUMENT, "ikrl_lmhead_status: null pointer");
  cudaStream_t s = as_stream(stream);
  int v = 0;
  IKRL_CUDA(cudaMemcpyAsync(&v, ws, sizeof(int), cudaMemcpyDeviceToHost, s));
  IKRL_CUDA(cudaStreamSynchronize(s));
  *status_out = v;
  if (v != 0) {
    set_error("device error 0x%x recorded by a tensor-core kernel (bounded wait expired)", v);
    return IKRL_ERR_DEVICE;
  }
  return IKRL_OK;
}

}  // extern "C"

// ---- allocation-free forward -------------------------------------------------------------------
//
// Some callers cannot allocate device memory at the moment they need log-probs: hosts that embed
// this library behind their own device-memory manager and forbid side allocations, frameworks
// that have already reserved all free memory in their caching pool (a cudaMalloc there fails or
// forces the pool to release memory and synchronise the device), and callers on a latency-critical
// path where an allocation's implicit synchronisation is not acceptable.  For them the forward
// below takes its scratch (the per-split row statistics and the device error word) from a fixed
// array compiled into the library instead of a caller-provided workspace.
//
// Limits and sharing rules:
//   * the array is kNoAllocScratchBytes (4 MiB) and lives on every GPU that loads the library
//     until the process exits; calls whose scratch would not fit are rejected with
//     IKRL_ERR_WORKSPACE (the message gives the sizes) -- use ikrl_lmhead_logprob_fwd instead;
//   * every call on a device uses the same array: calls whose kernels may overlap on the GPU
//     (different streams without ordering) race on it, so order them on one stream;
//   * the array keeps whatever the last call left in it; the error word at its start is cleared
//     by every call, the rest is fully rewritten before it is read;
//   * a bounded wait that expires inside a tensor-core kernel records a code in that error word
//     and the outputs become NaN; ikrl_lmhead_noalloc_status reads the word of the current device;
//   * the first call on each device looks up the device addresses of the library's two static
//     arrays (this scratch and the pacing counters of the wide kernel) with cudaGetSymbolAddress,
//     with that device current; make that first call before any stream capture begins.

namespace ikrl {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device, looked up once per device.  The
// same first call also resolves the pacing array, so that no later call on this device needs a
// symbol lookup, whatever its sizes.
int noalloc_scratch(void** out) {
  int dev = 0;
  IKRL_CUDA(cudaGetDevice(&dev));
  IKRL_REQUIRE(dev >= 0 && dev < kMaxDevices, IKRL_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    unsigned* pace = nullptr;
    int rc = pace_array(&pace);
    if (rc) return rc;
    void* p = nullptr;
    IKRL_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return IKRL_OK;
}

}  // namespace
}  // namespace ikrl

extern "C" int ikrl_lmhead_logprob_fwd_noalloc(const void* hidden, const void* weight, const int64_t* ids,
                                               int64_t N, int32_t H, int32_t V, float* logp, float* lse,
                                               void* stream) {
  clear_error();
  int rc = check_common(hidden, weight, ids, N, H, V, "ikrl_lmhead_logprob_fwd_noalloc");
  if (rc) return rc;
  const size_t need = ikrl_lmhead_fwd_workspace_bytes(N, H, V);
  IKRL_REQUIRE(need <= kNoAllocScratchBytes, IKRL_ERR_WORKSPACE,
               "ikrl_lmhead_logprob_fwd_noalloc: N=%lld rows (H=%d, V=%d) need %zu bytes of scratch, more than the "
               "built-in %zu; split the rows or call ikrl_lmhead_logprob_fwd with a workspace",
               (long long)N, H, V, need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if ((rc = noalloc_scratch(&scratch))) return rc;
  return ikrl_lmhead_logprob_fwd(hidden, weight, ids, N, H, V, logp, lse, scratch, kNoAllocScratchBytes, stream);
}

extern "C" int ikrl_lmhead_noalloc_status(int32_t* status_out, void* stream) {
  clear_error();
  IKRL_REQUIRE(status_out != nullptr, IKRL_ERR_INVALID_ARGUMENT, "ikrl_lmhead_noalloc_status: null pointer");
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return ikrl_lmhead_status(scratch, status_out, stream);
}
