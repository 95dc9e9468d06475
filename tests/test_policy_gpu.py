"""PolicyModel drop-in (invokerl/policy.py:60-196) on a small random-init Qwen3: per-token
log-probs, the shift and position-0 pad, the FSDP (materialised logits) branch, and the head's
gradients, against the fp32 oracle."""

from __future__ import annotations

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

V = 151936


def _tiny_qwen3(device):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    cfg = Qwen3Config(vocab_size=V, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=64, rope_theta=1e6,
                      max_position_embeddings=1024, tie_word_embeddings=True, use_cache=False)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(cfg).to(device=device, dtype=torch.bfloat16)
    model.train()
    model.gradient_checkpointing_enable()
    return model


def _batch(device, B=4, T=96):
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, V, (B, T), generator=g)
    lens = torch.randint(T // 2, T + 1, (B,), generator=g)
    am = torch.arange(T)[None, :] < lens[:, None]
    return ids.to(device), am.to(device)


@pytest.fixture(scope="module")
def setup():
    dev = torch.device("cuda")
    model = _tiny_qwen3(dev)
    ids, am = _batch(dev)
    return model, ids, am


def _oracle_lp(model, ids, am):
    with torch.no_grad():
        h = model.model(input_ids=ids, attention_mask=am).last_hidden_state[:, :-1]
    return oracle.lmhead_logprob(h.cpu(), model.lm_head.weight.detach().cpu(), ids[:, 1:].cpu())


def test_forward_matches_oracle(setup):
    from invokerl_b200.policy import PolicyModel

    model, ids, am = setup
    pm = PolicyModel.from_model(model, device=ids.device)
    lp = pm.forward(ids, am)
    assert lp.shape == ids.shape and lp.dtype == torch.float32
    assert torch.all(lp[:, 0] == 0)
    want = _oracle_lp(model, ids, am)
    torch.testing.assert_close(lp[:, 1:].detach().cpu(), want, rtol=0, atol=2e-3)
    lp2 = pm.forward_no_grad(ids, am)
    assert not lp2.requires_grad
    torch.testing.assert_close(lp2, lp.detach(), rtol=0, atol=0)


def test_fsdp_branch_matches_oracle(setup):
    from invokerl_b200.policy import PolicyModel

    model, ids, am = setup
    pm = PolicyModel.from_model(model, device=ids.device, fsdp_wrapped=True)
    with torch.no_grad():
        lp = pm.forward(ids, am)
    assert torch.all(lp[:, 0] == 0)
    want = _oracle_lp(model, ids, am)
    # logits are materialised in bf16 here (the reference's FSDP branch), so bf16 rounding of each
    # logit is added to the fused path's error
    torch.testing.assert_close(lp[:, 1:].cpu(), want, rtol=0, atol=3e-2)


def test_head_gradients_match_oracle(setup):
    from invokerl_b200.policy import PolicyModel

    model, ids, am = setup
    pm = PolicyModel.from_model(model, device=ids.device)
    with torch.no_grad():
        h = model.model(input_ids=ids, attention_mask=am).last_hidden_state[:, :-1].contiguous()
    h = h.clone().requires_grad_(True)
    w = model.lm_head.weight.detach().clone().requires_grad_(True)
    tgt = ids[:, 1:].contiguous()
    g = torch.Generator().manual_seed(2)
    up = torch.randn(tgt.shape, generator=g)
    lp = PolicyModel._chunk_ce_fn(w, h, tgt)
    (lp * up.to(lp.device)).sum().backward()
    lp_o, dh_o, dw_o = oracle.lmhead_logprob_grads(h.detach().cpu(), w.detach().cpu(), tgt.cpu(), up)
    torch.testing.assert_close(lp.detach().cpu(), lp_o, rtol=0, atol=2e-3)

    def rel(a, b):
        return float((a.float().cpu() - b).norm() / b.norm().clamp_min(1e-30))

    assert rel(h.grad, dh_o) <= 1e-2
    assert rel(w.grad, dw_o) <= 1e-2


def test_training_step_reaches_every_parameter(setup):
    """One GRPO step through forward -> loss -> backward: the tied embedding / LM-head weight and
    the transformer layers all receive finite gradients."""
    from invokerl_b200.algorithms import GRPO, RolloutBatch
    from invokerl_b200.policy import PolicyModel

    model, ids, am = setup
    B, T = ids.shape
    pm = PolicyModel.from_model(model, device=ids.device)
    with torch.no_grad():
        base = pm.forward(ids, am)
    g = torch.Generator(device=ids.device).manual_seed(3)
    resp = am.clone()
    resp[:, : T // 4] = False
    batch = RolloutBatch(token_ids=ids, prompt_mask=am & ~resp, response_mask=resp, attention_mask=am,
                         rewards=torch.tensor([1.0, 0.0, 1.0, 1.0], device=ids.device), token_rewards=None,
                         old_log_probs=base + 0.05 * torch.randn(B, T, device=ids.device, generator=g),
                         ref_log_probs=base + 0.1 * torch.randn(B, T, device=ids.device, generator=g),
                         group_ids=torch.zeros(B, dtype=torch.long, device=ids.device), group_size=4)
    algo = GRPO(clip_eps=0.2, beta=0.04)
    model.zero_grad(set_to_none=True)
    adv = algo.compute_advantages(batch)
    loss, metrics = algo.compute_loss(pm.forward(ids, am), batch, adv)
    loss.backward()
    assert torch.isfinite(loss)
    for name, p in model.named_parameters():
        assert p.grad is not None, name
        assert torch.isfinite(p.grad).all(), name
    assert float(model.lm_head.weight.grad.float().norm()) > 0
    model.zero_grad(set_to_none=True)
