/*
 * invokerl_b200 — C ABI of the B200 (sm_100a) kernels behind invokerl's training hot path.
 *
 * The hot path is invokerl's per-token log-prob computation (invokerl/policy.py:60-196) and
 * the advantage/loss hooks of its algorithms (invokerl/algorithms/{base,grpo,dapo,ppo,simpo}.py).
 * The reference is pure Python over PyTorch; the Python package `invokerl_b200` binds these
 * entry points through ctypes and keeps the reference's Python interface.  Every entry point
 * below names the reference code it replaces.
 *
 * Conventions (all entry points):
 *   - Plain device pointers, sizes and a `cudaStream_t` passed as `void* stream`; every launch is
 *     ordered on that stream and nothing synchronises the host unless the comment says so.
 *   - The library allocates no device memory: outputs and workspaces belong to the caller.  A
 *     `*_workspace_bytes` function gives the workspace size where one is needed.
 *   - Static device state: two file-scope arrays in the library's device code, present on every
 *     GPU that loads it.  (1) The pacing counters of the 256x512 K1 kernel (512 x 4 bytes): every
 *     paced launch on a device zeroes and uses them, so paced launches that overlap on two streams
 *     weaken each other's pacing; the waits are bounded and the results do not depend on it.
 *     (2) The 4 MiB scratch of ikrl_lmhead_logprob_fwd_noalloc (below); no other entry point
 *     touches it.
 *   - Return value: IKRL_OK (0) or an IKRL_ERR_* code; `ikrl_last_error()` then holds a message
 *     (thread-local).  No C++ exception crosses this boundary.
 *   - Row-major tensors.  Masks are bool tensors read as bytes (0 / non-zero).
 */
#ifndef INVOKERL_B200_H_
#define INVOKERL_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define IKRL_API __attribute__((visibility("default")))
#else
#define IKRL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  IKRL_OK = 0,
  IKRL_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative or inconsistent size */
  IKRL_ERR_ALIGNMENT = 2,        /* pointer or stride misses the alignment a kernel needs */
  IKRL_ERR_UNSUPPORTED = 3,      /* dtype / shape combination the kernels do not cover */
  IKRL_ERR_WORKSPACE = 4,        /* workspace missing or smaller than *_workspace_bytes() */
  IKRL_ERR_CUDA = 5,             /* a CUDA runtime/driver call failed (message has the name) */
  IKRL_ERR_DEVICE = 6            /* a kernel recorded a device-side fault (bounded wait expired) */
};

enum { IKRL_DTYPE_F32 = 0, IKRL_DTYPE_BF16 = 1 };

/* KL estimators of invokerl/algorithms/grpo.py:117-123. */
enum { IKRL_KL_SCHULMAN = 0, IKRL_KL_SIMPLE = 1, IKRL_KL_NONE = 2 };

/* Loss families that share the clipped-ratio kernel. */
enum {
  IKRL_LOSS_GRPO = 0, /* grpo.py:84-143 and dapo.py:90-150: L = sum((pl + beta*kl)*m)/n */
  IKRL_LOSS_PPO = 1   /* ppo.py:108-184: L = pl_mean + vf_coef*vf + entropy term + kl term */
};

/* Number of doubles in the per-call sum vector (`sums`) of the clipped-ratio loss. */
#define IKRL_LOSS_NSUMS 16
/* Number of floats in the metrics vector of the clipped-ratio loss. */
#define IKRL_LOSS_NMETRICS 12
/* Number of floats in the metrics vector of SimPO. */
#define IKRL_SIMPO_NMETRICS 8

/* ---- library ---------------------------------------------------------------------------- */

/* Last error message of the calling thread ("" when none). */
IKRL_API const char* ikrl_last_error(void);
/* ABI version; bumps whenever a signature below changes. */
IKRL_API int ikrl_abi_version(void);
/* Number of kernels this library has launched in this process (host-side counter). */
IKRL_API unsigned long long ikrl_launch_count(void);

/* ---- launch tuning ------------------------------------------------------------------------- */
/* Process-wide launch choices of the tensor-core (K1) and loss (K3) kernels.  Each knob has a
 * fixed default, the configuration the library is measured and shipped with; the library reads
 * no environment variable.  The other values exist for A/B timing, and every value is covered by
 * a GPU parity test.  A knob affects the calls made after it is set; set knobs before launches
 * that should see them, not concurrently with calls on other host threads.  No counterpart in the
 * reference (its arithmetic is PyTorch's). */
enum {
  IKRL_TUNE_CTA_PAIRS = 0,      /* K1: 1 CTA pairs, tcgen05 cta_group::2 (default); 0 single CTAs */
  IKRL_TUNE_SKIP_ZERO_ROWS = 1, /* K1 backward: 1 skip rows whose upstream gradient is 0 (default);
                                   0 process every row (no host synchronisation) */
  IKRL_TUNE_WIDE = 2,           /* K1 pair tile: -1 auto (default: 256x512 when K >= 1024, and the
                                   256x256 tile for dH when it balances better); 0 never 256x512;
                                   1 always; 2 the K >= 1024 rule without the dH balance choice */
  IKRL_TUNE_PERSISTENT = 3,     /* K1 pair kernels: 1 one resident pair per two SMs (default);
                                   0 one pair per work unit */
  IKRL_TUNE_PACE = 4,           /* 256x512 kernel: which launches pace their persistent pairs, a
                                   mask: 1 forward, 2 dS recompute, 4 dH (and a one-chunk bf16
                                   dW), 8 fp32 dW; 15 all; 0 none; -1 auto (default): all but a
                                   forward with K < 2048 */
  IKRL_TUNE_PACE_KB = 5,        /* K blocks between pacing checkpoints (default 128) */
  IKRL_TUNE_PACE_LAG = 6,       /* checkpoints a pair may lead the slowest by (default 1) */
  IKRL_TUNE_BALANCE_SPLITS = 7, /* K1 dS launches: 1 pick the vocab split count for balance of
                                   the persistent pairs (default); 0 the L2 rule alone */
  IKRL_TUNE_L2_POLICY = 8,      /* 256x512 kernel L2 hints, 10*a + b for the A and B loads, each
                                   0 normal / 1 evict-last / 2 evict-first; -1 default (a=1, b=0) */
  IKRL_TUNE_L2_BUDGET_MB = 9,   /* L2 megabytes the vocab split rule gives the resident hidden
                                   rows; 0 auto (default: 40 when H >= 2048, else 24) */
  IKRL_TUNE_LOSS_KERNEL = 10,   /* GRPO/DAPO loss: 1 register loads (default); 2 bulk-copy staged;
                                   0 the general clipped-ratio kernel */
  IKRL_TUNE_PACE_KB_LONG = 11,  /* pacing checkpoint spacing of the dW and dH launches (default 128) */
  IKRL_TUNE_SPLIT_TAIL = 12,    /* 256x512 kernel: how many of each tile's last K blocks (0-4) run
                                   first-half-first, so the epilogue drains the first accumulator
                                   half under the second half's last MMAs; default 4; 0 halves
                                   interleaved to the end */
  IKRL_TUNE_DH_SPLIT_K = 13,    /* K1 backward dH with few row tiles: -1 auto (default: split the
                                   vocabulary reduction into K ranges summed in a fixed order when
                                   the 256x512 tiles alone leave pairs idle); 0 or 1 never; n > 1
                                   n ranges wherever the partial buffer holds them */
  IKRL_TUNE_COUNT = 14
};
/* Passed as `value`, restores the knob's default. */
#define IKRL_TUNE_DEFAULT (-0x7fffffffffffffffLL - 1)
/* Sets `knob` to `value` (IKRL_ERR_INVALID_ARGUMENT outside its range); the old value goes to
 * *previous when that is not NULL. */
IKRL_API int ikrl_set_tuning(int32_t knob, int64_t value, int64_t* previous);
IKRL_API int ikrl_get_tuning(int32_t knob, int64_t* value);

/* ---- K3: advantages ------------------------------------------------------------------------ */

/* Count of non-zero mask bytes -> *count_out (int64, device).  Feeds num_tokens =
 * mask.sum().clamp(min=1) of grpo.py:127, dapo.py:105, ppo.py:121; with rows sharded over ranks
 * the caller all-reduces this count before the loss.  Sets *count_out (no accumulation). */
IKRL_API int ikrl_mask_count(const uint8_t* mask, int64_t n, int64_t* count_out, void* stream);

/* Default credit assignment of invokerl/algorithms/base.py:86-110:
 * adv[b,t] = rewards[b] * mask[b,t]. */
IKRL_API int ikrl_broadcast_advantages(const float* rewards, const uint8_t* response_mask, int32_t B,
                              int32_t T, float* adv_out, void* stream);

/* Group-normalised sequence advantages, invokerl/algorithms/grpo.py:72-80 and
 * dapo.py:55-88.  Groups are G contiguous rows (rewards.view(-1, G)); std is unbiased and
 * clamped to >= 1e-8 (G == 1 gives NaN, as torch.std does).
 *   filter_zero_var != 0: DAPO dynamic sampling, adv *= (std > 1e-8)          (dapo.py:69-74)
 *   truncated != NULL  : adv = overlong_penalty where truncated[b]            (dapo.py:82-86)
 * adv_out[b,t] = adv[b] * mask[b,t].  Optional row_adv_out[B] receives adv[b]. */
IKRL_API int ikrl_group_advantages(const float* rewards, const uint8_t* response_mask,
                          const uint8_t* truncated, int32_t B, int32_t T, int32_t G,
                          int32_t filter_zero_var, float overlong_penalty, float* adv_out,
                          float* row_adv_out, void* stream);

/* Token-level group normalisation of grpo.py:62-70: per (group, position) mean and unbiased
 * std over the G rows of token_rewards, adv = (tr - mean) / max(std, 1e-8) * mask. */
IKRL_API int ikrl_token_group_advantages(const float* token_rewards, const uint8_t* response_mask,
                                int32_t B, int32_t T, int32_t G, float* adv_out, void* stream);

/* Masked mean and unbiased std of x over mask (ppo.py:123-127 whitening) -> out[0]=mean,
 * out[1]=std, out[2]=count (float).  count < 2 leaves whitening off (out[3] = 0, else 1). */
IKRL_API size_t ikrl_masked_moments_workspace_bytes(int64_t n);
IKRL_API int ikrl_masked_moments(const float* x, const uint8_t* mask, int64_t n, float* out4, void* ws,
                        size_t ws_bytes, void* stream);

/* PPO generalised advantage estimation, invokerl/algorithms/ppo.py:80-106: one reverse scan per
 * row.  rewards_bt != NULL uses token rewards; otherwise the sequence reward rewards_b[b] is
 * placed at the last response token of row b.  values[b,t] are the value predictions.
 * adv_out[b,t] = gae[b,t] * mask[b,t]. */
IKRL_API int ikrl_gae_advantages(const float* rewards_b, const float* rewards_bt, const float* values,
                        const uint8_t* response_mask, int32_t B, int32_t T, float gamma,
                        float lam, float* adv_out, void* stream);

/* ---- K3: clipped-ratio loss (GRPO / DAPO / PPO) ------------------------------------------- */

typedef struct {
  int32_t family;        /* IKRL_LOSS_GRPO or IKRL_LOSS_PPO */
  float ratio_lo;        /* clamp lower bound: 1 - clip_eps (GRPO/PPO) or 1 - clip_eps_low */
  float ratio_hi;        /* clamp upper bound: 1 + clip_eps (GRPO/PPO) or 1 + clip_eps_high */
  float clip_metric_eps; /* clip_frac counts |ratio - 1| > clip_metric_eps */
  float beta;            /* KL coefficient (0 disables the KL term and its gradient) */
  int32_t kl_type;       /* IKRL_KL_* */
  float entropy_coef;    /* PPO entropy bonus coefficient */
  float vf_coef;         /* PPO value-loss coefficient */
  float vf_clip_eps;     /* PPO value clipping */
} ikrl_loss_params;

/* Workspace of ikrl_clip_loss_fwd for n = B*T tokens. */
IKRL_API size_t ikrl_clip_loss_workspace_bytes(int64_t n_tokens);

/* One pass over the tokens of grpo.py:103-128 / dapo.py:108-128 / ppo.py:123-164.
 * Inputs [B,T]: new_lp (fp32 or bf16, `lp_dtype`), old_lp, adv (fp32), mask (bytes);
 * ref_lp (fp32, may be NULL when beta == 0); rewards [B] (for the "reward" metric and, with
 * G > 0, the zero-variance group count of dapo.py:132-135).
 * ntok: global token count (int64, device; max(ntok,1) is the normaliser n).
 * whiten: NULL or the 4 floats of ikrl_masked_moments (PPO advantage whitening).
 * values / old_values: NULL or [B,T] fp32 (PPO value loss, ppo.py:147-156).
 * Outputs: dlp_out [B,T] (dtype of new_lp; NULL skips it) = d loss / d new_lp for an upstream
 * gradient of 1;
 * dvalues_out: NULL or [B,T] fp32 gradient of the value loss;
 * sums_out[IKRL_LOSS_NSUMS] (double, device): the sums of this call's rows, reduced in a fixed
 * order (bitwise reproducible): 0 pl*m, 1 kl*m, 2 clipped*m, 3 0.5*log_ratio^2*m,
 * 4 sum of adv over masked tokens, 5 m, 6 lp*m, 7 value-loss max*m, 8 (pl+beta*kl)*m,
 * 9 sum(rewards), 10 B, 11 zero-variance groups, 12 groups, 13-15 zero.  With rows sharded over
 * ranks the caller all-reduces sums_out (SUM) before ikrl_clip_loss_finalize. */
IKRL_API int ikrl_clip_loss_fwd(const void* new_lp, int32_t lp_dtype, const float* old_lp,
                                const float* ref_lp, const float* adv, const uint8_t* mask,
                                const float* rewards, int32_t B, int32_t T, int32_t G,
                                const int64_t* ntok, const float* whiten, const float* values,
                                const float* old_values, const ikrl_loss_params* params,
                                void* dlp_out, float* dvalues_out, double* sums_out, void* ws,
                                size_t ws_bytes, void* stream);

/* Turns sums into the loss value (loss_out[0]) and the metrics of grpo.py:131-141 /
 * dapo.py:137-148 / ppo.py:170-182: metrics_out[IKRL_LOSS_NMETRICS] = loss, reward, kl,
 * policy_loss, clip_frac, approx_kl, advantages_mean, entropy, vf_loss, num_tokens,
 * zero_var_groups, num_groups.  One block of one launch; no host synchronisation. */
IKRL_API int ikrl_clip_loss_finalize(const double* sums, const int64_t* ntok,
                                     const ikrl_loss_params* params, float* loss_out,
                                     float* metrics_out, void* stream);

/* In-place g *= *scale (device scalar); returns at once on the device when *scale == 1.
 * The backward of every loss above: d(upstream * loss)/d lp. */
IKRL_API int ikrl_scale_grad(void* g, int32_t dtype, int64_t n, const float* scale, void* stream);

/* ---- K3: SimPO (invokerl/algorithms/simpo.py:48-90) -------------------------------------- */

/* Per-row masked mean of lp, pairwise -logsigmoid(beta*(chosen - rejected) - gamma), mean.
 * loss_out[0]; metrics_out[IKRL_SIMPO_NMETRICS]: loss, reward, chosen_reward, rejected_reward,
 * reward_accuracy, margin, avg_log_prob, num_pairs.  row_coef_out[B] = d loss / d lp[b,t] for
 * masked tokens of row b (upstream 1).  B must be even.  rewards may be NULL ("reward" = 0). */
IKRL_API size_t ikrl_simpo_workspace_bytes(int32_t B);
IKRL_API int ikrl_simpo_fwd(const void* lp, int32_t lp_dtype, const uint8_t* mask, const float* rewards,
                   int32_t B, int32_t T, float beta, float gamma, int32_t chosen_first,
                   float* loss_out, float* metrics_out, float* row_coef_out, void* ws,
                   size_t ws_bytes, void* stream);

/* dlp[b,t] = row_coef[b] * mask[b,t] * (*scale). */
IKRL_API int ikrl_simpo_bwd(const float* row_coef, const uint8_t* mask, int32_t B, int32_t T,
                   const float* scale, void* dlp_out, int32_t dlp_dtype, void* stream);

/* ---- K3: DPO (invokerl/algorithms/dpo.py:51-106) ----------------------------------------------- */

/* Per-row masked sum of (lp - ref_lp), pairwise -logsigmoid(beta*(chosen - rejected)) with label
 * smoothing, mean over pairs.  loss_out[0]; metrics_out[IKRL_SIMPO_NMETRICS]: loss, reward,
 * chosen_reward, rejected_reward, reward_accuracy, margin, 0, num_pairs.  row_coef_out[B] =
 * d loss / d lp[b,t] on masked tokens (upstream 1); the backward is ikrl_simpo_bwd. */
IKRL_API size_t ikrl_dpo_workspace_bytes(int32_t B);
IKRL_API int ikrl_dpo_fwd(const void* lp, int32_t lp_dtype, const float* ref_lp, const uint8_t* mask,
                          const float* rewards, int32_t B, int32_t T, float beta,
                          float label_smoothing, int32_t chosen_first, float* loss_out,
                          float* metrics_out, float* row_coef_out, void* ws, size_t ws_bytes,
                          void* stream);

/* ---- K2: logits -> log-prob (unfused path) ------------------------------------------------ */

/* Replaces -F.cross_entropy(logits, targets, reduction="none") of invokerl/policy.py:100-104
 * and :151-155 (and the chunk of :187-191).  logits bf16 [N, ld] (row stride ld >= V, in
 * elements), ids int64 [N] in [0, V).
 * logp[N] fp32 = logits[r, ids[r]] - logsumexp(logits[r, :V]); lse[N] fp32 (saved for the
 * backward); tgt_logit (nullable) = the gathered raw logit, bit-exact. */
IKRL_API int ikrl_logits_logprob_fwd(const void* logits, int64_t ld, const int64_t* ids, int64_t N,
                            int32_t V, float* logp, float* lse, float* tgt_logit, void* stream);

/* Backward of the above: dlogits[r, v] = dlogp[r] * ([v == ids[r]] - exp(logits[r,v] - lse[r]))
 * in bf16, row stride ld_out.  Rows with dlogp == 0 are written as zeros without reading. */
IKRL_API int ikrl_logits_logprob_bwd(const void* logits, int64_t ld, const int64_t* ids, const float* lse,
                            const float* dlogp, int64_t N, int32_t V, void* dlogits,
                            int64_t ld_out, void* stream);

/* ---- K1: fused LM-head log-prob (tcgen05 / TMEM / TMA) --------------------------------------- */

/* Replaces the LM head + cross-entropy of invokerl/policy.py:124-191 (`_chunked_lm_head_ce`,
 * `_chunk_ce_fn`): hidden bf16 [N, H] (row stride H), weight bf16 [V, H] (row stride H),
 * ids int64 [N] in [0, V) (-100 = ignored row, log p = -0.0).  logp[N] fp32 =
 * (h W^T)[r, ids[r]] - logsumexp_v (h W^T)[r, v]; lse[N] fp32 (nullable) is saved for the
 * backward.  The [N, V] logits never exist in memory.  H must be a multiple of 8; pointers
 * 16-byte aligned; the workspace 256-byte aligned. */
IKRL_API size_t ikrl_lmhead_fwd_workspace_bytes(int64_t N, int32_t H, int32_t V);
IKRL_API int ikrl_lmhead_logprob_fwd(const void* hidden, const void* weight, const int64_t* ids,
                                     int64_t N, int32_t H, int32_t V, float* logp, float* lse,
                                     void* ws, size_t ws_bytes, void* stream);

/* Backward of the above for upstream dlogp[N] fp32: dhidden bf16 [N, H] (nullable) and dweight
 * [V, H] (nullable; IKRL_DTYPE_BF16 or IKRL_DTYPE_F32, the latter optionally accumulated into).
 * Rows are processed in chunks of `chunk_rows` (<= 0: all rows at once); the workspace holds one
 * chunk of bf16 dlogits [chunk, round_up(V, 64)] plus, for a bf16 dweight over several chunks,
 * an fp32 [V, H] accumulator, plus the row-compaction buffers below, plus fp32 partials for a
 * dhidden split into K ranges (min(128M, 16 * min(N, chunk) * H) elements; see
 * IKRL_TUNE_DH_SPLIT_K).  A chunk's dhidden is then the fixed-order sum of its partials, so its
 * rounding depends on the number of ranges, which depends on the chunk's active rows.
 * Rows whose dlogp is exactly zero (tokens outside the loss mask) and ignore_index rows add
 * exact zeros to both gradients; they are left out of the GEMMs: the other rows are gathered
 * in order into a dense block (a copy of their hidden rows, [N, H] bf16 at most), and dhidden
 * is scattered back with zero rows elsewhere.  Choosing the chunks then needs the active-row
 * count on the host: the call synchronises `stream` once.  Inside a stream capture, or with
 * IKRL_TUNE_SKIP_ZERO_ROWS set to 0, all rows are processed and the call does not
 * synchronise.  With N = 0 a non-accumulated dweight is zeroed and nothing else runs. */
IKRL_API size_t ikrl_lmhead_bwd_workspace_bytes(int64_t N, int32_t H, int32_t V, int64_t chunk_rows,
                                                int32_t dweight_dtype, int32_t accumulate_dweight);
IKRL_API int ikrl_lmhead_logprob_bwd(const void* hidden, const void* weight, const int64_t* ids,
                                     const float* lse, const float* dlogp, int64_t N, int32_t H,
                                     int32_t V, int64_t chunk_rows, void* dhidden, void* dweight,
                                     int32_t dweight_dtype, int32_t accumulate_dweight, void* ws,
                                     size_t ws_bytes, void* stream);

/* Logit cache: the same forward and backward (invokerl/policy.py:124-191 and its autograd), with
 * the backward's logits recompute replaced by stored softmax numerators where memory allows.  The
 * reference recomputes every chunk's logits under torch.utils.checkpoint; here the forward can
 * store, for up to `cache_rows` rows, each 32-column chunk's numerators 2^(S log2e - m) in bf16
 * relative to the chunk maximum m, and m (fp32, log2 units); the backward then forms those rows'
 * dS = g (onehot - numerator 2^(m - lse log2e)) with a memory-bound pass instead of a GEMM, and
 * recomputes only the active rows without a slot.  Results equal the uncached calls up to the
 * bf16 rounding of the numerators (the same relative precision as the bf16 dS itself).
 *
 * Cache storage, owned by the caller, per slot: ikrl_lmhead_cache_row_elems gives q_elems bf16
 * (cache_q rows, 16-byte aligned) and m_elems fp32 (cache_m rows).  Forward: rows with
 * cache_mask[r] != 0 (every row when cache_mask is NULL) and a target other than -100 get slots
 * 0, 1, ... in row order until cache_rows are used; cache_slot[N] receives each row's slot or -1.
 * Workspace: ikrl_lmhead_cache_fwd_workspace_bytes.  Backward: pass the forward's cache_slot,
 * cache_q and cache_m, unchanged since; workspace and synchronisation as ikrl_lmhead_logprob_bwd
 * (inside a stream capture, or with IKRL_TUNE_SKIP_ZERO_ROWS = 0, the cache is not used and every
 * row is recomputed).  V must be a multiple of 8.  No counterpart in the reference. */
IKRL_API int ikrl_lmhead_cache_row_elems(int32_t V, int64_t* q_elems, int64_t* m_elems);
IKRL_API size_t ikrl_lmhead_cache_fwd_workspace_bytes(int64_t N, int32_t H, int32_t V);
IKRL_API int ikrl_lmhead_logprob_fwd_cached(const void* hidden, const void* weight, const int64_t* ids,
                                            int64_t N, int32_t H, int32_t V, float* logp, float* lse,
                                            const uint8_t* cache_mask, int64_t cache_rows,
                                            int32_t* cache_slot, void* cache_q, float* cache_m, void* ws,
                                            size_t ws_bytes, void* stream);
IKRL_API int ikrl_lmhead_logprob_bwd_cached(const void* hidden, const void* weight, const int64_t* ids,
                                            const float* lse, const float* dlogp, int64_t N, int32_t H,
                                            int32_t V, int64_t chunk_rows, void* dhidden, void* dweight,
                                            int32_t dweight_dtype, int32_t accumulate_dweight,
                                            const int32_t* cache_slot, const void* cache_q,
                                            const float* cache_m, void* ws, size_t ws_bytes, void* stream);

/* Allocation-free variant of ikrl_lmhead_logprob_fwd.  It has no counterpart in the reference.
 * For callers that cannot allocate device memory when they need log-probs: hosts whose own
 * allocator owns all device memory and forbids side allocations, or frameworks whose caching pool
 * has already reserved the free memory.  The scratch comes from a 4 MiB array built into the
 * library, held on every GPU that loads it until exit.  Calls needing more scratch (above 31,772
 * rows at H = 4096, 61,672 at H = 1024, V = 151936) fail with IKRL_ERR_WORKSPACE before any GPU
 * work.  All calls on a device share the array and it keeps the last call's contents (each call
 * clears what must start at zero), so calls that overlap on the GPU race.  The first call on a
 * device looks up the device addresses of the library's static arrays and should come before any
 * stream capture. */
IKRL_API int ikrl_lmhead_logprob_fwd_noalloc(const void* hidden, const void* weight,
                                             const int64_t* ids, int64_t N, int32_t H, int32_t V,
                                             float* logp, float* lse, void* stream);
/* Device status word of the last ikrl_lmhead_logprob_fwd_noalloc call on the current device
 * (synchronises `stream`): IKRL_OK, or IKRL_ERR_DEVICE with *status_out = the code a tensor-core
 * kernel recorded when a bounded wait expired (its outputs are then NaN).  No counterpart in the
 * reference. */
IKRL_API int ikrl_lmhead_noalloc_status(int32_t* status_out, void* stream);

/* Selects the K1 GEMM kernel for later calls in this process: CTA pairs (tcgen05 cta_group::2,
 * clusters of two; the default) or single CTAs (enable = 0).  Returns the previous setting.  The
 * same switch as ikrl_set_tuning(IKRL_TUNE_CTA_PAIRS, ...). */
IKRL_API int ikrl_lmhead_set_cta_pairs(int32_t enable);

/* The launch plan the K1 calls would use, for inspection and tests; makes no CUDA call.  gemm:
 * 0 the forward over `rows` rows, 1 the dS recompute of a backward chunk of `rows` rows, 2 its
 * dW (fp32 accumulator), 3 its dH undivided, 4 the K ranges of that dH.  num_sms: SMs of the GPU
 * (148 on B200; one persistent CTA pair per two).  plan_out[4] = kernel (0 single CTAs 128 x 256,
 * 1 CTA pairs 256 x 256, 2 wide CTA pairs 256 x 512), column tiles, tiles per work unit, work
 * units per row pair; for gemm 4, plan_out[0] = the K ranges (1: undivided; more: the 256 x 512
 * kernel stores fp32 partials that a second kernel sums) and the rest 0.  It follows the same
 * tuning knobs as the launches.  No counterpart in the reference. */
IKRL_API int ikrl_lmhead_plan(int32_t gemm, int64_t rows, int32_t H, int32_t V, int32_t num_sms,
                              int32_t* plan_out);

/* ---- vocab-parallel LM head ---------------------------------------------------------------- */
/* The LM head with W split along the vocabulary over P ranks (rows replicated), the optional
 * tensor-parallel layout of the hot path.  No counterpart in the reference, which keeps the whole
 * W on every rank; the results equal ikrl_lmhead_logprob_fwd/_bwd on the whole W.
 *
 * Forward on one rank: weight_shard holds vocabulary rows [vocab_start, vocab_start + V_shard).
 * Writes lse_shard[N] = logsumexp over the shard and tlogit[N] = the raw logit of ids[r] when the
 * id falls in the shard, -inf otherwise.  Workspace: ikrl_lmhead_fwd_workspace_bytes(N, H,
 * V_shard).  The caller gathers every rank's [tlogit; lse_shard] ([2, N] fp32, rank-major
 * [P, 2, N]) and calls ikrl_vocab_parallel_combine for logp[N] and the global lse[N]. */
IKRL_API int ikrl_lmhead_shard_fwd(const void* hidden, const void* weight_shard, const int64_t* ids, int64_t N,
                                   int32_t H, int32_t V_shard, int64_t vocab_start, float* tlogit, float* lse_shard,
                                   void* ws, size_t ws_bytes, void* stream);
IKRL_API int ikrl_vocab_parallel_combine(const float* parts, const int64_t* ids, int64_t N, int32_t P,
                                         int64_t V_total, float* logp, float* lse, void* stream);
/* Backward on one rank from the global lse: dweight_shard [V_shard, H] is this rank's slice of
 * dW (no communication), dhidden_partial [N, H] bf16 this rank's term of dH; the caller sums the
 * terms over ranks (all-reduce).  Same row skipping, workspace and synchronisation as
 * ikrl_lmhead_logprob_bwd with V = V_shard. */
IKRL_API int ikrl_lmhead_shard_bwd(const void* hidden, const void* weight_shard, const int64_t* ids,
                                   const float* lse, const float* dlogp, int64_t N, int32_t H, int32_t V_shard,
                                   int64_t vocab_start, int64_t chunk_rows, void* dhidden_partial,
                                   void* dweight_shard, int32_t dweight_dtype, int32_t accumulate_dweight, void* ws,
                                   size_t ws_bytes, void* stream);

/* ---- rollout packing ------------------------------------------------------------------------ */

/* Pads B variable-length rollouts into [B, T] tensors; replaces the per-row host loop of
 * invokerl/generator.py:414-455 (`VLLMGenerator._pack_output`).  Row b's token ids are
 * ids_flat[id_offsets[b] .. id_offsets[b+1]) and its log-probs lps_flat[lp_offsets[b] ..
 * lp_offsets[b+1]) (device CSR arrays, offsets int64 [B+1]).  Writes token_ids int64 (pad_id
 * after the sequence), log_probs fp32 (0 after the row's list), prompt_mask [0, prompt_len),
 * response_mask [prompt_len, prompt_len + completion_len) and attention_mask [0, seq_len) as
 * bytes; lengths past T are clipped like Python slices.  B <= 65535. */
IKRL_API int ikrl_pack_rollouts(const int64_t* ids_flat, const int64_t* id_offsets, const float* lps_flat,
                                const int64_t* lp_offsets, const int32_t* prompt_lens,
                                const int32_t* completion_lens, int32_t B, int32_t T, int64_t pad_id,
                                int64_t* token_ids, float* log_probs, uint8_t* prompt_mask,
                                uint8_t* response_mask, uint8_t* attention_mask, void* stream);

/* Device status word of the last K1 call that used workspace `ws` (synchronises `stream`):
 * IKRL_OK, or IKRL_ERR_DEVICE with *status_out = the recorded code (a bounded wait expired). */
IKRL_API int ikrl_lmhead_status(const void* ws, int32_t* status_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* INVOKERL_B200_H_ */
