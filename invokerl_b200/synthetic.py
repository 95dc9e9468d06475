"""Seeded synthetic inputs in the shapes and value distributions of the benchmark workloads.

There is no dataset on this path: rollouts are synthetic (prompt / completion spans, Bernoulli
rewards, log-probs drawn as -Exp(1) with Gaussian perturbations), hidden states are N(0, 1) and
LM-head weights N(0, 0.02).  Everything is generated on the CPU from a torch.Generator so the
same seed gives the same tensors on any machine with this torch version.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .algorithms.base import RolloutBatch

VOCAB = 151936


def rollout_batch(
    n_prompts: int,
    group_size: int,
    T: int,
    *,
    prompt_len: tuple[int, int] = (64, 256),
    completion_len: tuple[int, int] = (32, 256),
    vocab: int = VOCAB,
    seed: int = 0,
    lp_dtype: torch.dtype = torch.float32,
) -> RolloutBatch:
    """A RolloutBatch: prompt at [0, p), completion at [p, p+c) (clipped to T), padding after;
    rewards ~ Bernoulli(0.5); new = -Exp(1), old = new + N(0, 0.05), ref = new + N(0, 0.1).
    `new_log_probs` is returned in extras["new_log_probs"]."""
    g = torch.Generator().manual_seed(seed)
    B = n_prompts * group_size
    p = torch.randint(prompt_len[0], prompt_len[1] + 1, (B,), generator=g)
    c = torch.randint(completion_len[0], completion_len[1] + 1, (B,), generator=g)
    p = p.clamp(max=T - 1)
    c = torch.minimum(c, T - p)
    pos = torch.arange(T)[None, :]
    prompt_mask = pos < p[:, None]
    response_mask = (pos >= p[:, None]) & (pos < (p + c)[:, None])
    attention_mask = prompt_mask | response_mask
    token_ids = torch.randint(0, vocab, (B, T), generator=g)
    rewards = torch.bernoulli(torch.full((B,), 0.5), generator=g)
    new = -torch.empty(B, T).exponential_(1.0, generator=g)
    old = new + 0.05 * torch.randn(B, T, generator=g)
    ref = new + 0.1 * torch.randn(B, T, generator=g)
    return RolloutBatch(
        token_ids=token_ids,
        prompt_mask=prompt_mask,
        response_mask=response_mask,
        attention_mask=attention_mask,
        rewards=rewards,
        token_rewards=None,
        old_log_probs=old,
        ref_log_probs=ref,
        group_ids=torch.arange(n_prompts).repeat_interleave(group_size),
        group_size=group_size,
        extras={"new_log_probs": new.to(lp_dtype)},
    )


@dataclass
class LMHeadInputs:
    hidden: torch.Tensor  # [N, H] bf16
    weight: torch.Tensor  # [V, H] bf16
    targets: torch.Tensor  # [N] int64


def lmhead_inputs(N: int, H: int, V: int = VOCAB, *, seed: int = 0, w_std: float = 0.02) -> LMHeadInputs:
    """hidden ~ N(0,1) (post-RMSNorm scale), W ~ N(0, w_std), targets uniform in [0, V)."""
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(N, H, generator=g).to(torch.bfloat16)
    w = (w_std * torch.randn(V, H, generator=g)).to(torch.bfloat16)
    t = torch.randint(0, V, (N,), generator=g)
    return LMHeadInputs(h, w, t)


def logits_inputs(N: int, V: int = VOCAB, *, seed: int = 0, std: float = 2.0, mask_p: float = 0.5):
    """bf16 logits ~ N(0, std), uniform targets, upstream N(0,1) times a Bernoulli(mask_p) mask."""
    g = torch.Generator().manual_seed(seed)
    logits = (std * torch.randn(N, V, generator=g)).to(torch.bfloat16)
    t = torch.randint(0, V, (N,), generator=g)
    up = torch.randn(N, generator=g) * torch.bernoulli(torch.full((N,), mask_p), generator=g)
    return logits, t, up
