"""PPO (invokerl/algorithms/ppo.py:22-184): GAE as one reverse-scan launch per batch,
masked whitening as a two-pass moments launch, and the clipped surrogate, entropy, clipped value
loss and optional k3 KL as the shared clipped-ratio kernel."""

from __future__ import annotations

from torch import Tensor

from .. import _native as N
from .. import ops
from .base import BaseAlgorithm, RolloutBatch


class PPO(BaseAlgorithm):
    def __init__(
        self,
        clip_eps: float = 0.2,
        vf_clip_eps: float = 0.2,
        vf_coef: float = 0.5,
        entropy_coef: float = 0.01,
        gae_gamma: float = 1.0,
        gae_lambda: float = 0.95,
        beta: float = 0.0,
        **kwargs,
    ):
        super().__init__(
            clip_eps=clip_eps,
            vf_coef=vf_coef,
            entropy_coef=entropy_coef,
            gae_gamma=gae_gamma,
            gae_lambda=gae_lambda,
            beta=beta,
            **kwargs,
        )
        self.clip_eps = clip_eps
        self.vf_clip_eps = vf_clip_eps
        self.vf_coef = vf_coef
        self.entropy_coef = entropy_coef
        self.gae_gamma = gae_gamma
        self.gae_lambda = gae_lambda
        self.beta = beta

    def compute_advantages(self, batch: RolloutBatch) -> Tensor:
        values = batch.extras.get("values")
        if values is None:
            return ops.broadcast_advantages(batch.rewards, batch.response_mask)
        if batch.token_rewards is not None:
            return ops.gae_advantages(None, batch.token_rewards, values, batch.response_mask, self.gae_gamma,
                                      self.gae_lambda)
        return ops.gae_advantages(batch.rewards, None, values, batch.response_mask, self.gae_gamma,
                                  self.gae_lambda)

    def _params(self) -> N.LossParams:
        return ops.make_loss_params(
            N.IKRL_LOSS_PPO, 1.0 - self.clip_eps, 1.0 + self.clip_eps, self.clip_eps, self.beta,
            N.IKRL_KL_SCHULMAN if self.beta > 0 else N.IKRL_KL_NONE, self.entropy_coef, self.vf_coef,
            self.vf_clip_eps,
        )

    def compute_loss(self, new_log_probs: Tensor, batch: RolloutBatch, advantages: Tensor):
        params = self._params()
        ntok = self._global_token_count(batch.response_mask)
        # advantage whitening over the whole batch's masked tokens (all ranks when row-sharded)
        whiten = self._global_moments(ops.masked_moments(advantages, batch.response_mask))
        values = batch.extras.get("values")
        old_values = batch.extras.get("old_values")
        if values is None or old_values is None:
            values = old_values = None
        loss, sums, ntok = ops.clip_ratio_loss(
            new_log_probs, batch.old_log_probs, batch.ref_log_probs if self.beta > 0 else None, advantages,
            batch.response_mask, batch.rewards, 0, params, ntok=ntok, whiten=whiten, values=values,
            old_values=old_values,
        )
        _, mt = ops.clip_loss_finalize(self._global_sums(sums), ntok, params)
        m = mt.tolist()
        metrics = {
            "loss": m[0],
            "reward": m[1],
            "policy_loss": m[3],
            "vf_loss": m[8] if values is not None else 0.0,
            "entropy": m[7],
            "clip_frac": m[4],
            "approx_kl": m[5],
            "advantages_mean": m[6],
        }
        if self.beta > 0:
            metrics["kl"] = m[2]
        return loss, metrics
