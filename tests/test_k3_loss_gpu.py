"""K3 parity on the GPU: the drop-in algorithms against the reference's golden outputs and the
CPU oracle (advantages, loss, metrics and d loss / d new_log_probs)."""

import pytest
import torch

import oracle
from helpers import ALGO_CASES, assert_metrics_close, load, make_batch
from invokerl_b200 import _native as N
from invokerl_b200 import ops
from invokerl_b200.algorithms import DAPO, DPO, GRPO, PPO, SimPO
from invokerl_b200.synthetic import rollout_batch

pytestmark = pytest.mark.gpu
DEV = "cuda"
CLS = {"grpo": GRPO, "dapo": DAPO, "ppo": PPO, "simpo": SimPO, "dpo": DPO}


def run(algo, batch, new_lp, scale=1.0):
    adv = algo.compute_advantages(batch)
    lp = new_lp.clone().requires_grad_(True)
    loss, metrics = algo.compute_loss(lp, batch, adv)
    (loss * scale).backward()
    torch.cuda.synchronize()
    return adv, loss.detach(), metrics, lp.grad


@pytest.mark.parametrize("name", ALGO_CASES)
def test_algorithms_match_reference_golden(name):
    g = load(name)
    algo = CLS[g["kind"]](**g["kwargs"])
    b = make_batch(g["batch"], DEV)
    adv, loss, metrics, grad = run(algo, b, g["new_lp"].to(DEV))
    out = g["out"]
    # advantages / loss: 1e-4 relative (fp32 accumulation)
    torch.testing.assert_close(adv.cpu(), out["adv"], rtol=1e-4, atol=1e-6, equal_nan=True)
    torch.testing.assert_close(loss.cpu().float(), out["loss"].float(), rtol=1e-4, atol=1e-6)
    assert_metrics_close(metrics, out["metrics"], rtol=1e-4, atol=1e-6)
    bf = g["new_lp"].dtype == torch.bfloat16
    assert grad.dtype == g["new_lp"].dtype
    torch.testing.assert_close(grad.cpu().float(), out["grad"].float(), rtol=1e-2 if bf else 1e-4,
                               atol=1e-7 if not bf else 1e-6)


def test_grpo_config1_against_oracle_many_seeds():
    for seed in range(5):
        b = rollout_batch(4, 4, 512, seed=100 + seed)
        nl = b.extras["new_log_probs"]
        adv_o = oracle.group_advantages(b.rewards, b.response_mask, 4)
        loss_o, met_o, g_o = oracle.clip_ratio_loss(nl, b.old_log_probs, b.ref_log_probs, adv_o, b.response_mask,
                                                    b.rewards)
        bd = make_batch(vars(b), DEV)
        adv, loss, metrics, grad = run(GRPO(), bd, nl.to(DEV))
        torch.testing.assert_close(adv.cpu(), adv_o, rtol=1e-4, atol=1e-6)
        assert abs(float(loss) - float(loss_o)) <= 1e-4 * abs(float(loss_o)) + 1e-6
        for k in ("kl", "policy_loss", "clip_frac", "approx_kl", "advantages_mean", "reward"):
            assert abs(metrics[k] - met_o[k]) <= 1e-4 * abs(met_o[k]) + 1e-6, k
        torch.testing.assert_close(grad.cpu(), g_o, rtol=1e-4, atol=1e-8)


def test_scaled_bandwidth_variant_against_oracle():
    """The HBM-sized variant of config 1 (B=1024 as 128x8, T=8192): size-independent checks and
    a full comparison with the oracle."""
    b = rollout_batch(128, 8, 8192, seed=7)
    nl = b.extras["new_log_probs"]
    bd = make_batch(vars(b), DEV)
    adv, loss, metrics, grad = run(GRPO(), bd, nl.to(DEV))
    adv_o = oracle.group_advantages(b.rewards, b.response_mask, 8)
    loss_o, met_o, g_o = oracle.clip_ratio_loss(nl, b.old_log_probs, b.ref_log_probs, adv_o, b.response_mask,
                                                b.rewards)
    torch.testing.assert_close(adv.cpu(), adv_o, rtol=1e-4, atol=1e-6)
    assert abs(float(loss) - float(loss_o)) <= 1e-4 * abs(float(loss_o)) + 1e-6
    torch.testing.assert_close(grad.cpu(), g_o, rtol=1e-4, atol=1e-9)
    # gradient is zero off the mask, exactly
    assert float(grad[~bd.response_mask].abs().max()) == 0.0


def test_sums_are_bitwise_reproducible():
    b = make_batch(vars(rollout_batch(16, 8, 1024, seed=9)), DEV)
    nl = rollout_batch(16, 8, 1024, seed=9).extras["new_log_probs"].to(DEV)
    algo = GRPO()
    adv = algo.compute_advantages(b)
    p = algo._params()
    outs = [ops.clip_ratio_loss(nl, b.old_log_probs, b.ref_log_probs, adv, b.response_mask, b.rewards, 8, p)[1]
            for _ in range(3)]
    assert all(torch.equal(outs[0], o) for o in outs[1:])


def test_upstream_scale_and_retain_graph():
    b0 = rollout_batch(4, 4, 256, seed=5)
    b = make_batch(vars(b0), DEV)
    nl = b0.extras["new_log_probs"].to(DEV)
    algo = GRPO()
    adv = algo.compute_advantages(b)
    lp = nl.clone().requires_grad_(True)
    loss, _ = algo.compute_loss(lp, b, adv)
    (loss * 0.25).backward(retain_graph=True)
    g1 = lp.grad.clone()
    lp.grad = None
    (loss * 2.0).backward()
    g2 = lp.grad.clone()
    torch.testing.assert_close(g2, g1 * 8.0, rtol=1e-6, atol=0)
    _, _, g_o = oracle.clip_ratio_loss(b0.extras["new_log_probs"], b0.old_log_probs, b0.ref_log_probs,
                                       adv.cpu(), b0.response_mask, b0.rewards)
    torch.testing.assert_close(g1.cpu(), g_o * 0.25, rtol=1e-4, atol=1e-9)


def test_no_grad_forward_skips_gradient_buffer():
    b0 = rollout_batch(2, 4, 128, seed=6)
    b = make_batch(vars(b0), DEV)
    algo = GRPO()
    with torch.no_grad():
        loss, m = algo.compute_loss(b0.extras["new_log_probs"].to(DEV), b, algo.compute_advantages(b))
    assert not loss.requires_grad and isinstance(m["loss"], float)


def test_gae_matches_oracle_long_rows():
    g = torch.Generator().manual_seed(3)
    B, T = 6, 3000
    mask = torch.rand(B, T, generator=g) < 0.7
    values = torch.randn(B, T, generator=g)
    rewards = torch.randn(B, generator=g)
    want = oracle.gae_advantages(rewards, None, values, mask, 0.99, 0.95)
    got = ops.gae_advantages(rewards.to(DEV), None, values.to(DEV), mask.to(DEV), 0.99, 0.95)
    torch.testing.assert_close(got.cpu(), want, rtol=1e-4, atol=1e-4)


def test_group_size_one_gives_nan_like_torch_std():
    r = torch.tensor([1.0, 0.0, 1.0], device=DEV)
    m = torch.ones(3, 4, dtype=torch.bool, device=DEV)
    adv = ops.group_advantages(r, m, 1)
    assert torch.isnan(adv).all()


@pytest.mark.parametrize("lean", ["2", "1", "0"])
@pytest.mark.parametrize("kl_type,lp_dtype", [("schulman", torch.float32), ("simple", torch.float32),
                                             ("schulman", torch.bfloat16)])
def test_grpo_kernel_variants_agree_with_oracle(lean, kl_type, lp_dtype):
    """The three GRPO loss kernels (bulk-copy staged, register loads, general clipped-ratio) on a
    batch of 23 full 1024-token tiles plus a 448-token partial tile."""
    with N.tuning(loss_kernel=int(lean)):
        _grpo_variant_case(kl_type, lp_dtype)


def _grpo_variant_case(kl_type, lp_dtype):
    b = rollout_batch(6, 4, 1000, prompt_len=(16, 200), completion_len=(100, 800), seed=77,
                      lp_dtype=lp_dtype)
    nl = b.extras["new_log_probs"]
    adv_o = oracle.group_advantages(b.rewards, b.response_mask, 4)
    loss_o, met_o, g_o = oracle.clip_ratio_loss(nl.float(), b.old_log_probs, b.ref_log_probs, adv_o,
                                                b.response_mask, b.rewards, kl_type=kl_type)
    bd = make_batch(vars(b), DEV)
    adv, loss, metrics, grad = run(GRPO(kl_type=kl_type), bd, nl.to(DEV))
    assert abs(float(loss) - float(loss_o)) <= 1e-4 * abs(float(loss_o)) + 1e-6
    for k in ("kl", "policy_loss", "clip_frac", "approx_kl", "advantages_mean", "reward"):
        assert abs(metrics[k] - met_o[k]) <= 1e-4 * abs(met_o[k]) + 1e-6, k
    bf = lp_dtype == torch.bfloat16
    torch.testing.assert_close(grad.cpu().float(), g_o.to(lp_dtype).float(), rtol=1e-2 if bf else 1e-4,
                               atol=1e-6 if bf else 1e-8)
