"""DPO (invokerl/algorithms/dpo.py:26-106): per-row masked sums of policy minus reference
log-probs, pairwise -logsigmoid margin with label smoothing, in two launches; the backward is one
broadcast launch."""

from __future__ import annotations

import torch
from torch import Tensor

from .. import ops
from .base import BaseAlgorithm, RolloutBatch


class DPO(BaseAlgorithm):
    def __init__(self, beta: float = 0.1, label_smoothing: float = 0.0, chosen_first: bool = True, **kwargs):
        super().__init__(beta=beta, label_smoothing=label_smoothing, **kwargs)
        self.beta = beta
        self.label_smoothing = label_smoothing
        self.chosen_first = chosen_first

    def compute_advantages(self, batch: RolloutBatch) -> Tensor:
        """DPO uses no advantages (dpo.py:47-49)."""
        return torch.zeros_like(batch.response_mask, dtype=torch.float32)

    def compute_loss(self, new_log_probs: Tensor, batch: RolloutBatch, advantages: Tensor):
        loss, mt = ops.dpo_loss(new_log_probs, batch.ref_log_probs, batch.response_mask, batch.rewards, self.beta,
                                self.label_smoothing, self.chosen_first)
        loss, mt = self._pair_share(loss, mt, new_log_probs.shape[0])
        m = mt.tolist()
        metrics = {
            "loss": m[0],
            "reward": m[1],
            "chosen_reward": m[2],
            "rejected_reward": m[3],
            "reward_accuracy": m[4],
            "margin": m[5],
        }
        return loss, metrics
