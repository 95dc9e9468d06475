"""CPU restatement of invokerl's hot-path arithmetic (ORACLE — test infrastructure only).

Each function names the reference lines it restates.  Arithmetic runs in float32 on the CPU,
like the reference's own fp32 path; autograd supplies the gradients the reference's autograd
would produce.  Not imported by the product package.
"""

from __future__ import annotations

import torch

__all__ = [
    "logprob_from_logits",
    "logprob_from_logits_grad",
    "lmhead_logprob",
    "lmhead_logprob_grads",
    "broadcast_advantages",
    "group_advantages",
    "token_group_advantages",
    "gae_advantages",
    "clip_ratio_loss",
    "simpo_loss",
    "dpo_loss",
    "pack_rollouts",
]


# ---- log-prob path: invokerl/policy.py ---------------------------------------------------------


def logprob_from_logits(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """log p(target) = x[target] - logsumexp(x) per row, in fp32.

    Restates ``-F.cross_entropy(logits, targets, reduction="none")`` of policy.py:100-104,
    :151-155 and :187-191 (logits upcast to fp32, the north-star precision)."""
    x = logits.float()
    lse = torch.logsumexp(x, dim=-1)
    tgt = torch.gather(x, -1, targets.long().unsqueeze(-1)).squeeze(-1)
    return tgt - lse


def logprob_from_logits_grad(logits: torch.Tensor, targets: torch.Tensor, upstream: torch.Tensor):
    """(log-probs, d(sum(upstream * lp))/d logits) by autograd of the fp32 restatement."""
    x = logits.detach().float().requires_grad_(True)
    lp = logprob_from_logits(x, targets)
    (lp * upstream.float()).sum().backward()
    return lp.detach(), x.grad


def lmhead_logprob(hidden: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor,
                   row_chunk: int = 4096) -> torch.Tensor:
    """F.linear(hidden, W) followed by the log-prob above (policy.py:173-191), fp32, processed in
    row chunks so the fp32 logits of a chunk are the only large temporary."""
    h = hidden.reshape(-1, hidden.shape[-1]).float()
    w = weight.float()
    t = targets.reshape(-1)
    out = torch.empty(h.shape[0], dtype=torch.float32)
    for s in range(0, h.shape[0], row_chunk):
        e = min(s + row_chunk, h.shape[0])
        out[s:e] = logprob_from_logits(h[s:e] @ w.t(), t[s:e])
    return out.reshape(targets.shape)


def lmhead_logprob_grads(hidden, weight, targets, upstream, row_chunk: int = 2048):
    """(lp, dH, dW) of sum(upstream * lp) for lp = lmhead_logprob(hidden, W, targets), fp32.

    The gradient is formed per row chunk as dlogits = g * (onehot - softmax), dH = dlogits W,
    dW = dlogits^T h — the autograd of policy.py:186-191 written out."""
    h = hidden.reshape(-1, hidden.shape[-1]).float()
    w = weight.float()
    t = targets.reshape(-1).long()
    g = upstream.reshape(-1).float()
    lp = torch.empty(h.shape[0], dtype=torch.float32)
    dh = torch.empty_like(h)
    dw = torch.zeros_like(w)
    for s in range(0, h.shape[0], row_chunk):
        e = min(s + row_chunk, h.shape[0])
        logits = h[s:e] @ w.t()
        lse = torch.logsumexp(logits, dim=-1, keepdim=True)
        p = torch.exp(logits - lse)
        lp[s:e] = torch.gather(logits, 1, t[s:e, None]).squeeze(1) - lse.squeeze(1)
        d = -p * g[s:e, None]
        d[torch.arange(e - s), t[s:e]] += g[s:e]
        dh[s:e] = d @ w
        dw += d.t() @ h[s:e]
    return lp.reshape(targets.shape), dh.reshape(hidden.shape), dw


# ---- advantages: invokerl/algorithms/{base,grpo,dapo,ppo}.py ------------------------------------


def broadcast_advantages(rewards: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """base.py:108-110: reward of the row on every response token."""
    return rewards.float()[:, None] * mask.float()


def _group_mean_std(x: torch.Tensor, G: int):
    g = x.float().reshape(-1, G, *x.shape[1:])
    mean = g.mean(dim=1, keepdim=True)
    std = g.std(dim=1, keepdim=True)  # unbiased, NaN for G == 1
    return g, mean, std


def group_advantages(rewards, mask, G, filter_zero_var=False, truncated=None, overlong_penalty=0.0):
    """grpo.py:72-80 (and dapo.py:61-88 with filter_zero_var / truncated)."""
    g, mean, std = _group_mean_std(rewards, G)
    adv = (g - mean) / std.clamp(min=1e-8)
    if filter_zero_var:
        adv = adv * (std > 1e-8).float()
    adv = adv.reshape(-1)
    if truncated is not None:
        adv = torch.where(truncated.bool(), torch.tensor(float(overlong_penalty)), adv)
    return adv[:, None] * mask.float()


def token_group_advantages(token_rewards, mask, G):
    """grpo.py:62-70: normalise token rewards per (group, position)."""
    g, mean, std = _group_mean_std(token_rewards, G)
    adv = ((g - mean) / std.clamp(min=1e-8)).reshape(token_rewards.shape)
    return adv * mask.float()


def gae_advantages(rewards, token_rewards, values, mask, gamma, lam):
    """ppo.py:80-106: reverse GAE scan per row; the sequence reward sits on the last response
    token when no token rewards are given."""
    m = mask.float()
    B, T = m.shape
    if token_rewards is not None:
        r = token_rewards.float()
    else:
        r = torch.zeros(B, T)
        for b in range(B):
            idx = torch.nonzero(mask[b]).flatten()
            if idx.numel():
                r[b, idx[-1]] = float(rewards[b])
    v = values.float()
    out = torch.zeros(B, T)
    carry = torch.zeros(B)
    for t in range(T - 1, -1, -1):
        nxt = v[:, t + 1] if t + 1 < T else torch.zeros(B)
        delta = r[:, t] + gamma * nxt - v[:, t]
        carry = delta + gamma * lam * carry * m[:, t]
        out[:, t] = carry
    return out * m


# ---- losses -------------------------------------------------------------------------------------


def clip_ratio_loss(new_lp, old_lp, ref_lp, adv, mask, rewards, *, family="grpo", clip_lo=0.2,
                    clip_hi=0.2, clip_metric_eps=None, beta=0.04, kl_type="schulman", G=0,
                    entropy_coef=0.0, vf_coef=0.5, vf_clip_eps=0.2, values=None, old_values=None):
    """GRPO / DAPO (grpo.py:103-141, dapo.py:102-148) and PPO (ppo.py:119-182) losses.

    Returns (loss, metrics dict, d loss / d new_lp) with the reference's metric keys."""
    lp = new_lp.detach().float().requires_grad_(True)
    m = mask.float()
    n = m.sum().clamp(min=1.0)
    a = adv.float()
    if family == "ppo":
        sel = a[mask.bool()]
        if sel.numel() > 1:
            a = (a - sel.mean()) / (sel.std() + 1e-8) * m
    log_ratio = lp - old_lp.float()
    ratio = torch.exp(log_ratio)
    s1 = ratio * a
    s2 = torch.clamp(ratio, 1.0 - clip_lo, 1.0 + clip_hi) * a
    pl = -torch.minimum(s1, s2)
    kl = None
    if ref_lp is not None and (family != "ppo" or beta > 0):
        d = ref_lp.float() - lp
        kl = torch.exp(d) - d - 1.0 if kl_type == "schulman" else -d
    eps_m = clip_lo if clip_metric_eps is None else clip_metric_eps
    metrics = {}
    if family == "ppo":
        plm = (pl * m).sum() / n
        entropy = -(lp * m).sum() / n
        vf = torch.tensor(0.0)
        if values is not None and old_values is not None:
            ret = a + old_values.float()
            vclip = old_values.float() + (values.float() - old_values.float()).clamp(-vf_clip_eps, vf_clip_eps)
            vf = 0.5 * (torch.maximum((values.float() - ret) ** 2, (vclip - ret) ** 2) * m).sum() / n
        loss = plm + vf_coef * vf - entropy_coef * entropy
        if beta > 0 and kl is not None:
            loss = loss + beta * (kl * m).sum() / n
        metrics.update(policy_loss=float(plm.detach()), vf_loss=float(vf.detach()), entropy=float(entropy.detach()))
        if beta > 0 and kl is not None:
            metrics["kl"] = float((kl.detach() * m).sum()) / float(n)
    else:
        loss = ((pl + beta * kl) * m).sum() / n
        metrics.update(kl=float((kl.detach() * m).sum()) / float(n),
                       policy_loss=float((pl.detach() * m).sum()) / float(n))
        if G:
            grp = rewards.float().reshape(-1, G)
            zv = int((grp.std(dim=1) < 1e-8).sum())
            metrics.update(zero_var_groups=zv, filtered_frac=zv / max(1, grp.shape[0]))
    with torch.no_grad():
        metrics.update(
            loss=float(loss.detach()),
            reward=float(rewards.float().mean()),
            clip_frac=float((((ratio - 1.0).abs() > eps_m).float() * m).sum()) / float(n),
            approx_kl=float(((0.5 * log_ratio ** 2) * m).sum()) / float(n),
            advantages_mean=float(a[mask.bool()].mean()) if mask.any() else 0.0,
        )
    loss.backward()
    return loss.detach(), metrics, lp.grad.to(new_lp.dtype)


def simpo_loss(new_lp, mask, rewards, beta=2.0, gamma=0.5, chosen_first=True):
    """simpo.py:59-90: length-normalised log-prob margin of chosen over rejected rows."""
    lp = new_lp.detach().float().requires_grad_(True)
    m = mask.float()
    avg = (lp * m).sum(dim=1) / m.sum(dim=1).clamp(min=1.0)
    c, r = (avg[0::2], avg[1::2]) if chosen_first else (avg[1::2], avg[0::2])
    margin = beta * (c - r) - gamma
    loss = -torch.nn.functional.logsigmoid(margin).mean()
    metrics = dict(
        loss=float(loss.detach()),
        reward=float(rewards.float().mean()),
        chosen_reward=float(c.detach().mean()),
        rejected_reward=float(r.detach().mean()),
        reward_accuracy=float((c > r).float().mean()),
        margin=float(margin.detach().mean()),
        avg_log_prob=float(avg.detach().mean()),
    )
    loss.backward()
    return loss.detach(), metrics, lp.grad.to(new_lp.dtype)


def dpo_loss(new_lp, ref_lp, mask, rewards, beta=0.1, label_smoothing=0.0, chosen_first=True):
    """dpo.py:62-106: pairwise sigmoid loss on the policy-minus-reference sequence log-ratios."""
    lp = new_lp.detach().float().requires_grad_(True)
    m = mask.float()
    lr = (lp * m).sum(dim=1) - (ref_lp.float() * m).sum(dim=1)
    c, r = (lr[0::2], lr[1::2]) if chosen_first else (lr[1::2], lr[0::2])
    margin = beta * (c - r)
    ls = torch.nn.functional.logsigmoid
    if label_smoothing > 0:
        loss = ((1 - label_smoothing) * -ls(margin) + label_smoothing * -ls(-margin)).mean()
    else:
        loss = -ls(margin).mean()
    with torch.no_grad():
        metrics = dict(
            loss=float(loss),
            reward=float(rewards.float().mean()),
            chosen_reward=float((beta * c).mean()),
            rejected_reward=float((beta * r).mean()),
            reward_accuracy=float((beta * c > beta * r).float().mean()),
            margin=float(margin.mean()),
        )
    loss.backward()
    return loss.detach(), metrics, lp.grad.to(new_lp.dtype)


# ---- rollout packing: invokerl/generator.py ------------------------------------------------------


def pack_rollouts(all_ids, all_lps, prompt_lens, completion_lens, pad_id):
    """Padded [B, T] token ids, log-probs and prompt / response / attention masks of ragged
    rollouts, T = the longest sequence (generator.py:414-455, `_pack_output`)."""
    B = len(all_ids)
    T = max((len(x) for x in all_ids), default=0)
    token_ids = torch.full((B, T), pad_id, dtype=torch.long)
    log_probs = torch.zeros(B, T, dtype=torch.float32)
    prompt_mask = torch.zeros(B, T, dtype=torch.bool)
    response_mask = torch.zeros(B, T, dtype=torch.bool)
    attention_mask = torch.zeros(B, T, dtype=torch.bool)
    for i in range(B):
        n = len(all_ids[i])
        token_ids[i, :n] = torch.tensor(all_ids[i], dtype=torch.long)
        m = min(len(all_lps[i]), T)
        log_probs[i, :m] = torch.tensor(all_lps[i][:m], dtype=torch.float32)
        p, c = prompt_lens[i], completion_lens[i]
        prompt_mask[i, :p] = True
        response_mask[i, p:p + c] = True
        attention_mask[i, :n] = True
    return dict(token_ids=token_ids, log_probs=log_probs, prompt_mask=prompt_mask, response_mask=response_mask,
                attention_mask=attention_mask)
