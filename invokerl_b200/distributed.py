"""Row sharding of the hot path across ranks (one process per GPU).

invokerl replicates every RolloutBatch on every rank (invokerl/distributed.py:236-302,
invokerl/trainer.py:131-140).  Here each rank takes whole prompt groups — G contiguous rows,
the layout of ``group_ids = arange(B/G).repeat_interleave(G)`` (trainer.py:317) — so group
advantages need no communication.  The only collectives of the path are the all-reduce of the
response-token count before the loss and of the metric sums after it (``algorithms.base``).
"""

from __future__ import annotations

import torch

from .algorithms.base import RolloutBatch


def group_shard_bounds(B: int, G: int, rank: int, world: int) -> tuple[int, int]:
    """Row range [start, end) of `rank`: whole groups, as even as possible, contiguous."""
    if G <= 0 or B % G:
        raise ValueError(f"B={B} is not a multiple of group_size={G}")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    ngroups = B // G
    base, extra = divmod(ngroups, world)
    g0 = rank * base + min(rank, extra)
    g1 = g0 + base + (1 if rank < extra else 0)
    return g0 * G, g1 * G


def shard_rows(x, start: int, end: int, B: int):
    if isinstance(x, torch.Tensor) and x.dim() >= 1 and x.shape[0] == B:
        return x[start:end]
    return x


def shard_batch(batch: RolloutBatch, rank: int, world: int) -> RolloutBatch:
    """This rank's whole groups of `batch` (views, no copies)."""
    B = batch.token_ids.shape[0]
    s, e = group_shard_bounds(B, batch.group_size, rank, world)
    return RolloutBatch(
        token_ids=batch.token_ids[s:e],
        prompt_mask=batch.prompt_mask[s:e],
        response_mask=batch.response_mask[s:e],
        attention_mask=batch.attention_mask[s:e],
        rewards=batch.rewards[s:e],
        token_rewards=None if batch.token_rewards is None else batch.token_rewards[s:e],
        old_log_probs=batch.old_log_probs[s:e],
        ref_log_probs=batch.ref_log_probs[s:e],
        group_ids=None if batch.group_ids is None else batch.group_ids[s:e],
        group_size=batch.group_size,
        weight_version=batch.weight_version,
        extras={k: shard_rows(v, s, e, B) for k, v in batch.extras.items()},
    )
