"""SimPO (invokerl/algorithms/simpo.py:23-90): per-row masked mean of the log-probs, pairwise
-logsigmoid margin and its gradient in two launches; the backward is one broadcast launch."""

from __future__ import annotations

import torch
from torch import Tensor

from .. import ops
from .base import BaseAlgorithm, RolloutBatch


class SimPO(BaseAlgorithm):
    def __init__(self, beta: float = 2.0, gamma: float = 0.5, chosen_first: bool = True, **kwargs):
        super().__init__(beta=beta, gamma=gamma, **kwargs)
        self.beta = beta
        self.gamma = gamma
        self.chosen_first = chosen_first

    def compute_advantages(self, batch: RolloutBatch) -> Tensor:
        """SimPO uses no advantages (simpo.py:44-46)."""
        return torch.zeros_like(batch.response_mask, dtype=torch.float32)

    def compute_loss(self, new_log_probs: Tensor, batch: RolloutBatch, advantages: Tensor):
        loss, mt = ops.simpo_loss(new_log_probs, batch.response_mask, batch.rewards, self.beta, self.gamma,
                                  self.chosen_first)
        loss, mt = self._pair_share(loss, mt, new_log_probs.shape[0])
        m = mt.tolist()
        metrics = {
            "loss": m[0],
            "reward": m[1],
            "chosen_reward": m[2],
            "rejected_reward": m[3],
            "reward_accuracy": m[4],
            "margin": m[5],
            "avg_log_prob": m[6],
        }
        return loss, metrics
