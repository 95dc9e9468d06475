"""Pin the CPU oracle against golden vectors produced by running the reference itself."""

import pytest
import torch

import oracle
from helpers import ALGO_CASES, assert_metrics_close, load

ORACLE_KW = {
    "grpo": lambda kw: dict(family="grpo", clip_lo=kw.get("clip_eps", 0.2), clip_hi=kw.get("clip_eps", 0.2),
                            beta=kw.get("beta", 0.04), kl_type=kw.get("kl_type", "schulman")),
    "dapo": lambda kw: dict(family="grpo", clip_lo=kw.get("clip_eps_low", 0.2),
                            clip_hi=kw.get("clip_eps_high", 0.28), beta=kw.get("beta", 0.04)),
    "ppo": lambda kw: dict(family="ppo", clip_lo=kw.get("clip_eps", 0.2), clip_hi=kw.get("clip_eps", 0.2),
                           beta=kw.get("beta", 0.0), entropy_coef=kw.get("entropy_coef", 0.01),
                           vf_coef=kw.get("vf_coef", 0.5), vf_clip_eps=kw.get("vf_clip_eps", 0.2)),
}


def oracle_advantages(kind, kw, b):
    m = b["response_mask"]
    G = b["group_size"]
    if kind == "grpo":
        if b["token_rewards"] is not None:
            return oracle.token_group_advantages(b["token_rewards"], m, G)
        return oracle.group_advantages(b["rewards"], m, G)
    if kind == "dapo":
        pen = kw.get("overlong_penalty", -1.0)
        tr = b["extras"].get("truncated") if pen != 0.0 else None
        return oracle.group_advantages(b["rewards"], m, G, filter_zero_var=kw.get("filter_zero_var", True),
                                       truncated=tr, overlong_penalty=pen)
    if kind == "ppo":
        v = b["extras"].get("values")
        if v is None:
            return oracle.broadcast_advantages(b["rewards"], m)
        return oracle.gae_advantages(b["rewards"], b["token_rewards"], v, m, kw.get("gae_gamma", 1.0),
                                     kw.get("gae_lambda", 0.95))
    return torch.zeros_like(m, dtype=torch.float32)


@pytest.mark.parametrize("name", ALGO_CASES)
def test_oracle_matches_reference_algorithms(name):
    g = load(name)
    kind, kw, b, out = g["kind"], g["kwargs"], g["batch"], g["out"]
    adv = oracle_advantages(kind, kw, b)
    torch.testing.assert_close(adv, out["adv"], rtol=1e-5, atol=1e-6, equal_nan=True)
    if kind == "simpo":
        loss, metrics, grad = oracle.simpo_loss(g["new_lp"], b["response_mask"], b["rewards"],
                                                beta=kw.get("beta", 2.0), gamma=kw.get("gamma", 0.5),
                                                chosen_first=kw.get("chosen_first", True))
    elif kind == "dpo":
        loss, metrics, grad = oracle.dpo_loss(g["new_lp"], b["ref_log_probs"], b["response_mask"], b["rewards"],
                                              beta=kw.get("beta", 0.1), label_smoothing=kw.get("label_smoothing", 0.0),
                                              chosen_first=kw.get("chosen_first", True))
    else:
        okw = ORACLE_KW[kind](kw)
        ex = b["extras"]
        loss, metrics, grad = oracle.clip_ratio_loss(
            g["new_lp"], b["old_log_probs"], b["ref_log_probs"], out["adv"], b["response_mask"], b["rewards"],
            G=b["group_size"] if kind == "dapo" else 0, values=ex.get("values"), old_values=ex.get("old_values"),
            **okw)
        if kind == "grpo":
            metrics.pop("zero_var_groups", None)
            metrics.pop("filtered_frac", None)
    torch.testing.assert_close(loss.float(), out["loss"].float(), rtol=1e-5, atol=1e-6)
    assert_metrics_close(metrics, out["metrics"], rtol=1e-5)
    bf = g["new_lp"].dtype == torch.bfloat16
    torch.testing.assert_close(grad.float(), out["grad"].float(), rtol=8e-3 if bf else 1e-5, atol=1e-7)


def test_oracle_matches_reference_logits_path():
    g = load("logits_small")
    lp, dx = oracle.logprob_from_logits_grad(g["logits"], g["targets"], g["upstream"])
    torch.testing.assert_close(lp, g["lp_fp32"], rtol=0, atol=1e-5)
    torch.testing.assert_close(dx, g["dlogits_fp32"], rtol=1e-4, atol=1e-6)
    # The reference's default (bf16) output is the fp32 value rounded to bf16.
    assert (lp.to(torch.bfloat16).float() - g["lp_bf16"].float()).abs().max() <= 0.0625


def test_oracle_matches_reference_lmhead_small():
    g = load("lmhead_small")
    lp, dh, dw = oracle.lmhead_logprob_grads(g["hidden"], g["weight"], g["targets"], g["upstream"])
    torch.testing.assert_close(lp, g["lp_fp32"], rtol=0, atol=1e-4)
    torch.testing.assert_close(dh, g["dh_fp32"], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(dw, g["dw_fp32"], rtol=1e-4, atol=1e-5)


def test_oracle_matches_reference_chunked_branch():
    from invokerl_b200.synthetic import lmhead_inputs

    g = load("lmhead_chunked_seed")
    B, T, H, V = g["shape"]
    li = lmhead_inputs(B * T, H, V, seed=g["seed"], w_std=g["w_std"])
    lp = oracle.lmhead_logprob(li.hidden, li.weight, li.targets).reshape(B, T)
    torch.testing.assert_close(lp, g["lp_fp32"], rtol=0, atol=2e-4)


def test_oracle_matches_reference_rollout_packing():
    g = load("rollout_pack")
    out = oracle.pack_rollouts(g["all_ids"], g["all_lps"], g["prompt_lens"], g["completion_lens"], g["pad_id"])
    for k in ("token_ids", "log_probs", "prompt_mask", "response_mask", "attention_mask"):
        assert out[k].dtype == g[k].dtype, k
        assert torch.equal(out[k], g[k]), k
