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

    def _pair_share(self, loss: Tensor, metrics: Tensor, rows: int) -> tuple[Tensor, Tensor]:
        """Pairwise losses (SimPO, DPO) over row shards of whole pairs: the loss and every metric are
        means over pairs, so this rank's loss becomes its share (local mean x local pairs / global
        pairs, which scales its gradient the same way) and the metrics become the global means
        (one all-reduce of the pair count, one of the pair-weighted metrics)."""
        if not self._sharded():
            return loss, metrics
        import torch.distributed as dist

        p_local = rows // 2
        p = torch.tensor([float(p_local)], dtype=torch.float64, device=metrics.device)
        dist.all_reduce(p, group=self.process_group)
        mt = metrics.double() * p_local
        dist.all_reduce(mt, group=self.process_group)
        # The pair count stays on the device (no host synchronisation); a batch with no pair on any
        # rank gives a zero loss share and zero metrics instead of a division by zero.
        pc = p.clamp(min=1.0)
        share = (p_local / pc).to(loss.dtype).reshape(())
        return loss * share, (mt / pc).float()

    def _global_moments(self, w: Tensor) -> Tensor:
        """[mean, unbiased std, count, enabled] over the whole batch from each rank's own
        (`ops.masked_moments`): one all-gather of (count, count * mean, M2) per rank, combined with
        the pairwise update of Chan et al. (M2 = sum M2_r + sum n_r (mean_r - mean)^2) in fp64."""
        if not self._sharded():
            return w
        import torch.distributed as dist

        w64 = w.double()
        n = w64[2]
        mean = torch.where(n > 0, w64[0], torch.zeros_like(n))
        m2 = torch.where(n > 1, w64[1] * w64[1] * (n - 1), torch.zeros_like(n))
        local = torch.stack([n, n * mean, m2])
        parts = [torch.empty_like(local) for _ in range(dist.get_world_size(self.process_group))]
        dist.all_gather(parts, local, group=self.process_group)
        allp = torch.stack(parts)
        nt = allp[:, 0].sum()
        mean_g = allp[:, 1].sum() / nt.clamp(min=1.0)
        means = torch.where(allp[:, 0] > 0, allp[:, 1] / allp[:, 0].clamp(min=1.0), mean_g)
        m2_g = allp[:, 2].sum() + (allp[:, 0] * (means - mean_g) ** 2).sum()
        on = nt > 1
        std_g = torch.where(on, torch.sqrt(m2_g / (nt - 1).clamp(min=1.0)), torch.full_like(nt, float("nan")))
        return torch.stack([mean_g, std_g, nt, on.double()]).float()

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
