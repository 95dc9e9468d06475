// Rollout packing: variable-length generated sequences into the padded [B, T] tensors of a
// RolloutBatch (invokerl/generator.py:414-455, GenerationOutput packing).
//
// The reference fills each row with a host-side torch.tensor(...) per sequence and per field and
// sets the masks by slicing, B times five small copies.  Here the host concatenates the ragged
// token ids and log-probs once (CSR: values + B+1 offsets), moves them in one copy each, and one
// launch writes every field of every row.
#include "common.cuh"

namespace ikrl {
namespace {

constexpr int kPackThreads = 256;

// One thread per (row, position): token id (pad after the sequence), log-prob (0 after the
// row's log-prob list), and the three masks.  Lengths past T are clipped like Python slices.
__global__ void __launch_bounds__(kPackThreads) pack_rollouts_kernel(
    const int64_t* __restrict__ ids_flat, const int64_t* __restrict__ id_offsets, const float* __restrict__ lps_flat,
    const int64_t* __restrict__ lp_offsets, const int32_t* __restrict__ prompt_lens,
    const int32_t* __restrict__ completion_lens, int32_t T, int64_t pad_id, int64_t* __restrict__ token_ids,
    float* __restrict__ log_probs, uint8_t* __restrict__ prompt_mask, uint8_t* __restrict__ response_mask,
    uint8_t* __restrict__ attention_mask) {
  const int64_t b = blockIdx.y;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= T) return;
  const int64_t i0 = id_offsets[b];
  const int64_t seq_len = id_offsets[b + 1] - i0;
  const int64_t l0 = lp_offsets[b];
  const int64_t lp_len = lp_offsets[b + 1] - l0;
  const int64_t pl = prompt_lens[b], cl = completion_lens[b];
  const int64_t o = b * T + j;
  token_ids[o] = j < seq_len ? ids_flat[i0 + j] : pad_id;
  log_probs[o] = j < lp_len ? lps_flat[l0 + j] : 0.f;
  prompt_mask[o] = j < pl ? 1 : 0;
  response_mask[o] = (j >= pl && j < pl + cl) ? 1 : 0;
  attention_mask[o] = j < seq_len ? 1 : 0;
}

}  // namespace
}  // namespace ikrl

using namespace ikrl;

extern "C" {

int ikrl_pack_rollouts(const int64_t* ids_flat, const int64_t* id_offsets, const float* lps_flat,
                       const int64_t* lp_offsets, const int32_t* prompt_lens, const int32_t* completion_lens,
                       int32_t B, int32_t T, int64_t pad_id, int64_t* token_ids, float* log_probs, uint8_t* prompt_mask,
                       uint8_t* response_mask, uint8_t* attention_mask, void* stream) {
  clear_error();
  IKRL_REQUIRE(B >= 0 && T >= 0, IKRL_ERR_INVALID_ARGUMENT, "ikrl_pack_rollouts: bad sizes B=%d T=%d", B, T);
  if (B == 0 || T == 0) return IKRL_OK;
  IKRL_REQUIRE(id_offsets && lp_offsets && prompt_lens && completion_lens && token_ids && log_probs && prompt_mask &&
                   response_mask && attention_mask,
               IKRL_ERR_INVALID_ARGUMENT, "ikrl_pack_rollouts: null pointer");
  IKRL_REQUIRE(B <= 65535, IKRL_ERR_UNSUPPORTED, "ikrl_pack_rollouts: B=%d above 65535 rows per call", B);
  const dim3 grid((unsigned)((T + kPackThreads - 1) / kPackThreads), (unsigned)B);
  pack_rollouts_kernel<<<grid, kPackThreads, 0, as_stream(stream)>>>(ids_flat, id_offsets, lps_flat, lp_offsets,
                                                                     prompt_lens, completion_lens, T, pad_id,
                                                                     token_ids, log_probs, prompt_mask,
                                                                     response_mask, attention_mask);
  return check_launch("pack_rollouts_kernel");
}

}  // extern "C"
