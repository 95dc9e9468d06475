"""GRPO (invokerl/algorithms/grpo.py:23-143) on the fused K3 kernels.

compute_advantages: one launch (group mean / unbiased std / broadcast over the mask).
compute_loss: a token-count launch, one fused ratio+clip+KL+masked-sum launch that also writes
d loss / d new_log_probs, one finalize launch, and a single device-to-host copy of the metrics
(the reference issues ~25 launches and 7 blocking .item() calls).
"""

from __future__ import annotations

from torch import Tensor

from .. import _native as N
from .. import ops
from .base import BaseAlgorithm, RolloutBatch


class GRPO(BaseAlgorithm):
    """Group Relative Policy Optimization; hyper-parameters as in grpo.py:32-42."""

    def __init__(self, clip_eps: float = 0.2, beta: float = 0.04, kl_type: str = "schulman", **kwargs):
        super().__init__(clip_eps=clip_eps, beta=beta, kl_type=kl_type, **kwargs)
        self.clip_eps = clip_eps
        self.beta = beta
        self.kl_type = kl_type

    def compute_advantages(self, batch: RolloutBatch) -> Tensor:
        G = batch.group_size
        if batch.token_rewards is not None:
            return ops.token_group_advantages(batch.token_rewards, batch.response_mask, G)
        return ops.group_advantages(batch.rewards, batch.response_mask, G)

    def _params(self) -> N.LossParams:
        return ops.make_loss_params(
            N.IKRL_LOSS_GRPO, 1.0 - self.clip_eps, 1.0 + self.clip_eps, self.clip_eps, self.beta, self.kl_type
        )

    def compute_loss(self, new_log_probs: Tensor, batch: RolloutBatch, advantages: Tensor):
        params = self._params()
        ntok = self._global_token_count(batch.response_mask)
        loss, sums, ntok = ops.clip_ratio_loss(
            new_log_probs, batch.old_log_probs, batch.ref_log_probs, advantages, batch.response_mask,
            batch.rewards, batch.group_size, params, ntok=ntok,
        )
        _, mt = ops.clip_loss_finalize(self._global_sums(sums), ntok, params)
        m = mt.tolist()  # the one device->host copy of the step
        metrics = {
            "loss": m[0],
            "reward": m[1],
            "kl": m[2],
            "policy_loss": m[3],
            "clip_frac": m[4],
            "approx_kl": m[5],
            "advantages_mean": m[6],
        }
        return loss, metrics
