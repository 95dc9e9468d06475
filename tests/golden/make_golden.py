"""Generate the golden fixtures of tests/golden/ by running the reference implementation.

Run in a container that has the reference checkout (invokerl, pure Python over PyTorch), naming
its root either way:

    python tests/golden/make_golden.py --reference <reference checkout>
    INVOKERL_REFERENCE=<reference checkout> python tests/golden/make_golden.py

Each case stores its seeded inputs (or, for the one large case, the seed that regenerates them)
and the reference's outputs: advantages, loss, metrics dict and d loss / d new_log_probs for the
algorithm hooks (invokerl/algorithms/*.py), and log-probs plus gradients for the log-prob path
(invokerl/policy.py).  The fixtures are small and committed; nothing at test time needs the
reference.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

def _reference_root() -> str:
    """Root of the reference checkout: --reference PATH, else $INVOKERL_REFERENCE; no default."""
    if "--reference" in sys.argv:
        i = sys.argv.index("--reference")
        if i + 1 >= len(sys.argv):
            raise SystemExit("--reference needs a path")
        root = sys.argv[i + 1]
        del sys.argv[i:i + 2]
    else:
        root = os.environ.get("INVOKERL_REFERENCE", "")
    if not root or not (Path(root) / "invokerl" / "policy.py").exists():
        raise SystemExit("name the reference checkout with --reference PATH or INVOKERL_REFERENCE=PATH "
                         "(the directory that contains invokerl/policy.py)")
    return root


REF = _reference_root()
if REF not in sys.path:
    sys.path.insert(0, REF)

from invokerl.algorithms import DAPO, DPO, GRPO, PPO, SimPO  # noqa: E402
from invokerl.algorithms import RolloutBatch as RefBatch  # noqa: E402
from invokerl.policy import PolicyModel  # noqa: E402

from invokerl_b200.synthetic import lmhead_inputs, logits_inputs, rollout_batch  # noqa: E402

torch.set_num_threads(os.cpu_count() or 1)


def to_ref(b) -> RefBatch:
    return RefBatch(
        token_ids=b.token_ids, prompt_mask=b.prompt_mask, response_mask=b.response_mask,
        attention_mask=b.attention_mask, rewards=b.rewards, token_rewards=b.token_rewards,
        old_log_probs=b.old_log_probs, ref_log_probs=b.ref_log_probs, group_ids=b.group_ids,
        group_size=b.group_size, extras={k: v for k, v in b.extras.items() if k != "new_log_probs"},
    )


def batch_dict(b) -> dict:
    return dict(
        token_ids=b.token_ids, prompt_mask=b.prompt_mask, response_mask=b.response_mask,
        attention_mask=b.attention_mask, rewards=b.rewards, token_rewards=b.token_rewards,
        old_log_probs=b.old_log_probs, ref_log_probs=b.ref_log_probs, group_ids=b.group_ids,
        group_size=b.group_size, extras=dict(b.extras),
    )


def run_algo(algo, b, new_lp):
    rb = to_ref(b)
    adv = algo.compute_advantages(rb)
    lp = new_lp.clone().requires_grad_(True)
    loss, metrics = algo.compute_loss(lp, rb, adv)
    loss.backward()
    return dict(adv=adv.detach(), loss=loss.detach(), metrics=metrics, grad=lp.grad.detach())


def save(name: str, **payload) -> None:
    path = HERE / f"{name}.pt"
    torch.save(payload, path)
    print(f"{name}: {path.stat().st_size / 1024:.1f} KiB")


def algo_cases() -> None:
    # Config-1 shapes: 4 prompts x group 4, T=512, fp32.
    b = rollout_batch(4, 4, 512, seed=1)
    nl = b.extras["new_log_probs"]
    save("grpo_cfg1", kind="grpo", kwargs=dict(clip_eps=0.2, beta=0.04), batch=batch_dict(b), new_lp=nl,
         out=run_algo(GRPO(clip_eps=0.2, beta=0.04), b, nl))

    # bf16 new log-probs and the "simple" KL estimator.
    b = rollout_batch(2, 4, 96, prompt_len=(8, 40), completion_len=(8, 56), seed=2, lp_dtype=torch.bfloat16)
    nl = b.extras["new_log_probs"]
    save("grpo_bf16_simplekl", kind="grpo", kwargs=dict(clip_eps=0.2, beta=0.1, kl_type="simple"),
         batch=batch_dict(b), new_lp=nl, out=run_algo(GRPO(clip_eps=0.2, beta=0.1, kl_type="simple"), b, nl))

    # Edge cases: an all-masked row, a zero-variance group (zero advantages, min ties), ratios
    # just inside and just outside both clamp bounds and exactly 1 (a ratio exactly at 1 +- eps
    # depends on the last ulp of exp, which differs between libraries, so it is not pinned).
    b = rollout_batch(2, 4, 32, prompt_len=(4, 8), completion_len=(8, 20), seed=3)
    b.response_mask[0] = False
    b.rewards[4:8] = 1.0
    nl = b.extras["new_log_probs"].clone()
    eps = 0.2
    r = torch.tensor([1.0 - eps - 1e-3, 1.0 - eps + 1e-3, 1.0, 1.0 + eps - 1e-3, 1.0 + eps + 1e-3, 0.5, 2.0])
    for row in (1, 2, 5):
        nl[row, 10:17] = b.old_log_probs[row, 10:17] + torch.log(r)
        b.response_mask[row, 10:17] = True
    nl[3, 12] = b.old_log_probs[3, 12]  # log ratio exactly 0
    save("grpo_edges", kind="grpo", kwargs=dict(clip_eps=eps, beta=0.04), batch=batch_dict(b), new_lp=nl,
         out=run_algo(GRPO(clip_eps=eps, beta=0.04), b, nl))

    # All rows masked out: num_tokens clamps to 1, advantages_mean is 0.
    b = rollout_batch(1, 4, 16, prompt_len=(4, 8), completion_len=(2, 4), seed=4)
    b.response_mask[:] = False
    nl = b.extras["new_log_probs"]
    save("grpo_allmasked", kind="grpo", kwargs=dict(), batch=batch_dict(b), new_lp=nl, out=run_algo(GRPO(), b, nl))

    # Token-level rewards (credit-assignment hook).
    b = rollout_batch(2, 4, 64, prompt_len=(8, 20), completion_len=(8, 40), seed=5)
    b.token_rewards = torch.randn(8, 64, generator=torch.Generator().manual_seed(55))
    nl = b.extras["new_log_probs"]
    save("grpo_token_rewards", kind="grpo", kwargs=dict(), batch=batch_dict(b), new_lp=nl,
         out=run_algo(GRPO(), b, nl))

    # DAPO with truncation penalties and a zero-variance group; and without the filter.
    b = rollout_batch(4, 4, 128, prompt_len=(8, 40), completion_len=(16, 88), seed=6)
    b.rewards[0:4] = 0.0
    b.extras["truncated"] = torch.tensor([i % 5 == 0 for i in range(16)])
    nl = b.extras["new_log_probs"]
    save("dapo_default", kind="dapo", kwargs=dict(), batch=batch_dict(b), new_lp=nl, out=run_algo(DAPO(), b, nl))
    save("dapo_nofilter", kind="dapo", kwargs=dict(filter_zero_var=False, clip_eps_high=0.3, beta=0.02),
         batch=batch_dict(b), new_lp=nl, out=run_algo(DAPO(filter_zero_var=False, clip_eps_high=0.3, beta=0.02), b, nl))

    # PPO with values (GAE + value loss + KL) and without (reward broadcast).
    b = rollout_batch(2, 4, 96, prompt_len=(8, 40), completion_len=(8, 56), seed=7)
    g = torch.Generator().manual_seed(77)
    b.extras["values"] = 0.5 * torch.randn(8, 96, generator=g)
    b.extras["old_values"] = b.extras["values"] + 0.3 * torch.randn(8, 96, generator=g)
    nl = b.extras["new_log_probs"]
    save("ppo_values", kind="ppo", kwargs=dict(beta=0.04, gae_gamma=0.99), batch=batch_dict(b), new_lp=nl,
         out=run_algo(PPO(beta=0.04, gae_gamma=0.99), b, nl))
    b2 = rollout_batch(2, 4, 96, prompt_len=(8, 40), completion_len=(8, 56), seed=8)
    nl2 = b2.extras["new_log_probs"]
    save("ppo_novalues", kind="ppo", kwargs=dict(), batch=batch_dict(b2), new_lp=nl2, out=run_algo(PPO(), b2, nl2))
    b3 = rollout_batch(2, 4, 96, prompt_len=(8, 40), completion_len=(8, 56), seed=9)
    b3.token_rewards = 0.1 * torch.randn(8, 96, generator=torch.Generator().manual_seed(99))
    b3.extras["values"] = 0.5 * torch.randn(8, 96, generator=torch.Generator().manual_seed(98))
    nl3 = b3.extras["new_log_probs"]
    save("ppo_token_rewards", kind="ppo", kwargs=dict(), batch=batch_dict(b3), new_lp=nl3,
         out=run_algo(PPO(), b3, nl3))

    # SimPO pairs.
    b = rollout_batch(4, 2, 64, prompt_len=(8, 20), completion_len=(8, 40), seed=10)
    nl = b.extras["new_log_probs"]
    save("simpo_default", kind="simpo", kwargs=dict(), batch=batch_dict(b), new_lp=nl, out=run_algo(SimPO(), b, nl))
    save("simpo_rejected_first", kind="simpo", kwargs=dict(beta=1.5, gamma=0.2, chosen_first=False),
         batch=batch_dict(b), new_lp=nl, out=run_algo(SimPO(beta=1.5, gamma=0.2, chosen_first=False), b, nl))

    # DPO pairs (dpo.py): default, label smoothing, rejected-first ordering.
    b = rollout_batch(4, 2, 64, prompt_len=(8, 20), completion_len=(8, 40), seed=17)
    nl = b.extras["new_log_probs"]
    save("dpo_default", kind="dpo", kwargs=dict(), batch=batch_dict(b), new_lp=nl, out=run_algo(DPO(), b, nl))
    save("dpo_smoothing", kind="dpo", kwargs=dict(beta=0.3, label_smoothing=0.1, chosen_first=False),
         batch=batch_dict(b), new_lp=nl,
         out=run_algo(DPO(beta=0.3, label_smoothing=0.1, chosen_first=False), b, nl))


def logprob_cases() -> None:
    # Unfused path: bf16 logits -> log-prob, fp32 oracle and the reference's default bf16 output.
    logits, t, up = logits_inputs(64, 1000, seed=11)
    x = logits.float().requires_grad_(True)
    lp32 = -torch.nn.functional.cross_entropy(x, t, reduction="none")
    (lp32 * up).sum().backward()
    lp_bf16 = -torch.nn.functional.cross_entropy(logits, t, reduction="none")
    save("logits_small", logits=logits, targets=t, upstream=up, lp_fp32=lp32.detach(), dlogits_fp32=x.grad,
         lp_bf16=lp_bf16)

    # Fused path restated by the reference: PolicyModel._chunk_ce_fn on fp32 copies.
    li = lmhead_inputs(2 * 40, 64, 1000, seed=12, w_std=0.5)
    h = li.hidden.reshape(2, 40, 64)
    tg = li.targets.reshape(2, 40)
    hf = h.float().requires_grad_(True)
    wf = li.weight.float().requires_grad_(True)
    lp = PolicyModel._chunk_ce_fn(wf, hf, tg)
    g = torch.randn(2, 40, generator=torch.Generator().manual_seed(13))
    (lp * g).sum().backward()
    lp_bf16 = PolicyModel._chunk_ce_fn(li.weight, h, tg)
    save("lmhead_small", hidden=h, weight=li.weight, targets=tg, upstream=g, lp_fp32=lp.detach(), dh_fp32=hf.grad,
         dw_fp32=wf.grad, lp_bf16=lp_bf16)

    # The reference's chunked branch (B*T*V*4 >= 2 GiB): full vocabulary, inputs regenerated from
    # the seed at test time (W alone is 9.7 MB in bf16).
    B, T, H, V, seed = 2, 1800, 32, 151936, 14
    li = lmhead_inputs(B * T, H, V, seed=seed, w_std=0.5)

    class _Head(torch.nn.Module):
        def __init__(self, w):
            super().__init__()
            self.weight = torch.nn.Parameter(w)
            self.out_features = w.shape[0]

        def forward(self, x):
            return torch.nn.functional.linear(x, self.weight)

    stub = PolicyModel.__new__(PolicyModel)
    stub.model = torch.nn.Module()
    stub.model.lm_head = _Head(li.weight.float())
    assert B * T * V * 4 >= 2 * 1024**3
    with torch.no_grad():
        lp = stub._chunked_lm_head_ce(li.hidden.float().reshape(B, T, H), li.targets.reshape(B, T), 64)
    save("lmhead_chunked_seed", shape=(B, T, H, V), seed=seed, w_std=0.5, lp_fp32=lp)


def policy_forward_case() -> None:
    # PolicyModel.forward (policy.py:60-122): shift, log-probs of ids[:,1:], zero at position 0,
    # on a tiny random-init Qwen3 (fp32 weights).
    from transformers import Qwen3Config, Qwen3ForCausalLM

    torch.manual_seed(15)
    cfg = Qwen3Config(vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=128,
                      tie_word_embeddings=True)
    model = Qwen3ForCausalLM(cfg).float().eval()
    pm = PolicyModel.__new__(PolicyModel)
    pm.model = model
    pm.device = "cpu"
    pm.dtype = torch.float32
    pm._autocast_dtype = None
    pm._fsdp_wrapped = False
    g = torch.Generator().manual_seed(16)
    ids = torch.randint(0, 512, (3, 24), generator=g)
    am = torch.ones(3, 24, dtype=torch.bool)
    with torch.no_grad():
        lp = pm.forward(ids, am)
    save("policy_forward_tiny", config=cfg.to_dict(), state_dict=model.state_dict(), token_ids=ids,
         attention_mask=am, lp=lp)


def rollout_pack_case() -> None:
    # VLLMGenerator._pack_output (generator.py:414-455) on ragged sequences: prompt + completion
    # token ids, log-probs 0 on the prompt, one log-prob list shorter than its sequence.
    from invokerl.generator import VLLMGenerator

    class _Tok:
        pad_token_id = 151643

    gen = VLLMGenerator.__new__(VLLMGenerator)
    gen.tokenizer = _Tok()
    g = torch.Generator().manual_seed(21)
    all_ids, all_lps, pls, cls, texts = [], [], [], [], []
    for i in range(7):
        p = int(torch.randint(1, 40, (1,), generator=g))
        c = int(torch.randint(0, 60, (1,), generator=g))
        ids = torch.randint(0, 151936, (p + c,), generator=g).tolist()
        lps = [0.0] * p + (-torch.empty(c).exponential_(1.0, generator=g)).tolist()
        if i == 3:
            lps = lps[: max(0, len(lps) - 5)]
        all_ids.append(ids)
        all_lps.append(lps)
        pls.append(p)
        cls.append(c)
        texts.append(f"completion {i}")
    out = gen._pack_output(all_ids, all_lps, pls, cls, texts)
    save("rollout_pack", all_ids=all_ids, all_lps=all_lps, prompt_lens=pls, completion_lens=cls, texts=texts,
         pad_id=_Tok.pad_token_id, token_ids=out.token_ids, log_probs=out.log_probs, prompt_mask=out.prompt_mask,
         response_mask=out.response_mask, attention_mask=out.attention_mask)


CASES = {"algo": algo_cases, "logprob": logprob_cases, "policy": policy_forward_case, "rollout": rollout_pack_case}

if __name__ == "__main__":
    # no arguments: every case; otherwise the named groups
    for name in sys.argv[1:] or list(CASES):
        CASES[name]()
