"""DAPO (invokerl/algorithms/dapo.py:22-150) on the GRPO kernels with asymmetric clipping,
the zero-variance group filter and the overlong penalty folded into the advantage launch."""

from __future__ import annotations

from torch import Tensor

from .. import _native as N
from .. import ops
from .base import BaseAlgorithm, RolloutBatch


class DAPO(BaseAlgorithm):
    def __init__(
        self,
        clip_eps_low: float = 0.2,
        clip_eps_high: float = 0.28,
        beta: float = 0.04,
        overlong_penalty: float = -1.0,
        filter_zero_var: bool = True,
        **kwargs,
    ):
        super().__init__(
            clip_eps_low=clip_eps_low,
            clip_eps_high=clip_eps_high,
            beta=beta,
            overlong_penalty=overlong_penalty,
            **kwargs,
        )
        self.clip_eps_low = clip_eps_low
        self.clip_eps_high = clip_eps_high
        self.beta = beta
        self.overlong_penalty = overlong_penalty
        self.filter_zero_var = filter_zero_var

    def compute_advantages(self, batch: RolloutBatch) -> Tensor:
        truncated = None
        if self.overlong_penalty != 0.0 and batch.extras.get("truncated") is not None:
            truncated = batch.extras["truncated"]
        return ops.group_advantages(
            batch.rewards, batch.response_mask, batch.group_size, filter_zero_var=self.filter_zero_var,
            truncated=truncated, overlong_penalty=self.overlong_penalty,
        )

    def _params(self) -> N.LossParams:
        return ops.make_loss_params(
            N.IKRL_LOSS_GRPO, 1.0 - self.clip_eps_low, 1.0 + self.clip_eps_high, self.clip_eps_low, self.beta,
            "schulman",
        )

    def compute_loss(self, new_log_probs: Tensor, batch: RolloutBatch, advantages: Tensor):
        params = self._params()
        ntok = self._global_token_count(batch.response_mask)
        loss, sums, ntok = ops.clip_ratio_loss(
            new_log_probs, batch.old_log_probs, batch.ref_log_probs, advantages, batch.response_mask,
            batch.rewards, batch.group_size, params, ntok=ntok,
        )
        _, mt = ops.clip_loss_finalize(self._global_sums(sums), ntok, params)
        m = mt.tolist()
        zero_var = int(round(m[10]))
        num_groups = int(round(m[11]))
        metrics = {
            "loss": m[0],
            "reward": m[1],
            "kl": m[2],
            "policy_loss": m[3],
            "clip_frac": m[4],
            "approx_kl": m[5],
            "zero_var_groups": zero_var,
            "filtered_frac": zero_var / max(1, num_groups),
            "advantages_mean": m[6],
        }
        return loss, metrics
