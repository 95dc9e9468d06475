"""Algorithm contract of invokerl (invokerl/algorithms/base.py:26-150), kept field for field.

`RolloutBatch` and `BaseAlgorithm` have the reference's names, fields, signatures and return
types, so a trainer written against invokerl calls these classes unchanged.  The default
credit assignment runs on the GPU through the native library.

Row sharding (an addition; the reference replicates the batch on every rank): constructed with
``row_sharded=True`` inside an initialised ``torch.distributed`` job, an algorithm treats its batch
as this rank's whole prompt groups, all-reduces the response-token count before the loss and the
metric sums after it, and returns the metrics of the global batch.  The returned loss tensor is
this rank's share (sum over ranks = the global loss), so gradients summed over ranks are the
gradients of the global loss.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass, field
from typing import Any

import torch
from torch import Tensor

from .. import ops


@dataclass
class RolloutBatch:
    """A batch of generated rollouts with rewards (invokerl/algorithms/base.py:26-62)."""

    token_ids: Tensor  # [B, T] int64
    prompt_mask: Tensor  # [B, T] bool
    response_mask: Tensor  # [B, T] bool
    attention_mask: Tensor  # [B, T] bool
    rewards: Tensor  # [B]
    token_rewards: Tensor | None  # [B, T] or None
    old_log_probs: Tensor  # [B, T]
    ref_log_probs: Tensor  # [B, T]
    group_ids: Tensor | None  # [B]
    group_size: int = 1
    weight_version: int = 0
    extras: dict[str, Any] = field(default_factory=dict)


class BaseAlgorithm(ABC):
    """Base class of the algorithms (invokerl/algorithms/base.py:70-150)."""

    def __init__(self, **kwargs):
        self.config = kwargs
        self.row_sharded = bool(kwargs.get("row_sharded", False))
        self.process_group = kwargs.get("process_group", None)

    # -- distributed helpers -----------------------------------------------------------------

    def _sharded(self) -> bool:
        return (
            self.row_sharded
            and torch.distributed.is_available()
            and torch.distributed.is_initialized()
            and torch.distributed.get_world_size(self.process_group) > 1
        )

    def _global_token_count(self, response_mask: Tensor) -> Tensor:
        """int64 [1] device tensor: response tokens of the whole batch (all ranks)."""
        n = ops.mask_count(response_mask)
        if self._sharded():
            torch.distributed.all_reduce(n, group=self.process_group)
        return n

    def _global_sums(self, sums: Tensor) -> Tensor:
        if self._sharded():
            sums = sums.clone()
            torch.distributed.all_reduce(sums, group=self.process_group)
        return sums

    # -- credit assignment -------------------------------------------------------------------

    def compute_advantages(self, batch: RolloutBatch) -> Tensor:
        """Sequence reward broadcast to the response tokens (base.py:86-110)."""
        return ops.broadcast_advantages(batch.rewards, batch.response_mask)

    @abstractmethod
    def compute_loss(
        self,
        new_log_probs: Tensor,
        batch: RolloutBatch,
        advantages: Tensor,
    ) -> tuple[Tensor, dict[str, float]]:
        ...

    def on_step_start(self, step: int) -> None:
        pass

    def on_step_end(self, step: int, metrics: dict) -> None:
        pass
