"""Shared test helpers: golden loading, batch reconstruction, comparisons."""

from __future__ import annotations

from pathlib import Path

import torch

GOLDEN = Path(__file__).resolve().parent / "golden"

ALGO_CASES = [
    "grpo_cfg1",
    "grpo_bf16_simplekl",
    "grpo_edges",
    "grpo_allmasked",
    "grpo_token_rewards",
    "dapo_default",
    "dapo_nofilter",
    "ppo_values",
    "ppo_novalues",
    "ppo_token_rewards",
    "simpo_default",
    "simpo_rejected_first",
    "dpo_default",
    "dpo_smoothing",
]


def load(name: str) -> dict:
    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)


def make_batch(d: dict, device="cpu"):
    from invokerl_b200.algorithms import RolloutBatch

    def mv(x):
        return x.to(device) if isinstance(x, torch.Tensor) else x

    return RolloutBatch(
        token_ids=mv(d["token_ids"]),
        prompt_mask=mv(d["prompt_mask"]),
        response_mask=mv(d["response_mask"]),
        attention_mask=mv(d["attention_mask"]),
        rewards=mv(d["rewards"]),
        token_rewards=mv(d["token_rewards"]),
        old_log_probs=mv(d["old_log_probs"]),
        ref_log_probs=mv(d["ref_log_probs"]),
        group_ids=mv(d["group_ids"]),
        group_size=d["group_size"],
        extras={k: mv(v) for k, v in d["extras"].items() if k != "new_log_probs"},
    )


def rel_close(a: float, b: float, rtol: float = 1e-4, atol: float = 1e-6) -> bool:
    if a != a and b != b:
        return True
    return abs(a - b) <= atol + rtol * abs(b)


def assert_metrics_close(got: dict, want: dict, rtol=1e-4, atol=1e-6):
    assert set(got) == set(want), (sorted(got), sorted(want))
    for k, v in want.items():
        assert rel_close(float(got[k]), float(v), rtol, atol), f"{k}: got {got[k]} want {v}"
