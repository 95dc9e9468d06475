"""The drop-in at the caller: invokerl's own `Trainer.train_step` (trainer.py:335-346) drives this
package's classes unchanged.

The reference package is imported from baseline/_ref (an unmodified copy of its invokerl/
directory, pure Python); the tests skip when that copy is absent.  One tiny random-init Qwen3
(fp32 weights) and one rollout batch are run through the reference trainer's train_step three
ways:

  (i)   the reference's PolicyModel and GRPO (its F.linear + cross_entropy head in fp32);
  (ii)  the reference's PolicyModel with its two head methods patched to this package's fused
        LM-head kernel (the patch a maintainer would apply), and this package's GRPO;
  (iii) this package's PolicyModel.from_model and GRPO.

Arms (ii) and (iii) feed the head's GEMMs bf16 copies of the hidden states and of W (the kernel's
tensor-core input type), so they are compared with the fp32 arm (i) at the north-star log-prob
tolerance (2e-3 absolute) and at tolerances that bf16 rounding of the head inputs leaves for the
loss and metrics (5e-3 relative) and for every parameter's gradient (1e-2 relative Frobenius).
Given the same log-probs, the algorithm itself must agree with the reference's GRPO to 1e-4
relative (loss, metrics, and d loss / d log-probs).
"""

from __future__ import annotations

import copy
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
REF_ROOT = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
V, G, T = 4096, 4, 64


@pytest.fixture(scope="module")
def ref():
    if not (REF_ROOT / "invokerl" / "trainer.py").exists():
        pytest.skip("the reference package is not in baseline/_ref")
    if str(REF_ROOT) not in sys.path:
        sys.path.insert(0, str(REF_ROOT))
    import invokerl.algorithms
    import invokerl.policy
    import invokerl.trainer

    return invokerl


def tiny_model():
    from transformers import Qwen3Config, Qwen3ForCausalLM

    cfg = Qwen3Config(vocab_size=V, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=32, tie_word_embeddings=False,
                      use_cache=False)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    return Qwen3ForCausalLM(cfg).float().to(DEV)


def ref_policy(ref, model):
    pm = ref.policy.PolicyModel.__new__(ref.policy.PolicyModel)
    pm.model, pm.device, pm.dtype = model, DEV, torch.float32
    pm.master_weights_fp32, pm._autocast_dtype, pm._fsdp_wrapped = False, None, False
    return pm


def make_trainer(ref, policy, algorithm):
    tr = ref.trainer.Trainer.__new__(ref.trainer.Trainer)
    tr.policy, tr.algorithm = policy, algorithm
    tr.config = SimpleNamespace(accumulation_steps=2)
    return tr


@pytest.fixture(scope="module")
def setup(ref):
    from invokerl_b200.synthetic import rollout_batch

    model = tiny_model()
    b = rollout_batch(2, G, T, prompt_len=(8, 24), completion_len=(16, 40), vocab=V, seed=3)
    with torch.no_grad():
        lp = ref_policy(ref, model).forward(b.token_ids.to(DEV), b.attention_mask.to(DEV)).cpu()
    g = torch.Generator().manual_seed(1)
    old = lp + 0.05 * torch.randn(lp.shape, generator=g)
    refl = lp + 0.1 * torch.randn(lp.shape, generator=g)
    # the batch as the reference's own RolloutBatch on the host; train_step moves it to the device
    batch = ref.algorithms.RolloutBatch(
        token_ids=b.token_ids, prompt_mask=b.prompt_mask, response_mask=b.response_mask,
        attention_mask=b.attention_mask, rewards=b.rewards, token_rewards=None, old_log_probs=old,
        ref_log_probs=refl, group_ids=b.group_ids, group_size=G)
    return model, batch


def run_arm(ref, model, batch, arm, monkeypatch):
    from invokerl_b200 import ops
    from invokerl_b200.algorithms import GRPO
    from invokerl_b200.policy import PolicyModel

    m = copy.deepcopy(model)
    if arm == "reference":
        policy, algo = ref_policy(ref, m), ref.algorithms.GRPO(clip_eps=0.2, beta=0.04)
    elif arm == "patched":
        def fused_chunked_lm_head_ce(self, hidden_states, targets, chunk_size):
            return ops.lmhead_logprob(hidden_states, self.model.lm_head.weight, targets)

        monkeypatch.setattr(ref.policy.PolicyModel, "_chunked_lm_head_ce", fused_chunked_lm_head_ce)
        monkeypatch.setattr(ref.policy.PolicyModel, "_chunk_ce_fn",
                            staticmethod(lambda w, h, t: ops.lmhead_logprob(h, w, t)))
        policy, algo = ref_policy(ref, m), GRPO(clip_eps=0.2, beta=0.04)
    else:
        policy, algo = PolicyModel.from_model(m, device=DEV, dtype=torch.float32), GRPO(clip_eps=0.2, beta=0.04)
    trainer = make_trainer(ref, policy, algo)
    loss, metrics = trainer.train_step(batch)
    torch.cuda.synchronize()
    with torch.no_grad():
        lp = policy.forward(batch.token_ids.to(DEV), batch.attention_mask.to(DEV)).float().cpu()
    grads = {n: p.grad.detach().float().cpu() for n, p in m.named_parameters() if p.grad is not None}
    monkeypatch.undo()
    return float(loss.detach()), metrics, grads, lp


def rel_fro(a, b):
    return float((a - b).norm() / b.norm().clamp(min=1e-30))


@pytest.mark.parametrize("arm", ["patched", "dropin"])
def test_reference_train_step_drives_the_drop_in(ref, setup, arm, monkeypatch):
    model, batch = setup
    loss_r, met_r, grads_r, lp_r = run_arm(ref, model, batch, "reference", monkeypatch)
    loss, met, grads, lp = run_arm(ref, model, batch, arm, monkeypatch)
    assert float((lp - lp_r).abs().max()) <= 2e-3
    assert abs(loss - loss_r) <= 5e-3 * abs(loss_r) + 1e-6
    assert set(met) == set(met_r)
    for k, v in met_r.items():
        assert abs(met[k] - v) <= 5e-3 * abs(v) + 1e-5, (k, met[k], v)
    assert set(grads) == set(grads_r) and len(grads) > 10  # every parameter of the model got a gradient
    for n, g in grads_r.items():
        assert rel_fro(grads[n], g) <= 1e-2, n


def test_drop_in_grpo_matches_reference_grpo_on_the_same_log_probs(ref, setup):
    """The algorithm alone, on identical inputs: this package's GRPO against the reference's."""
    from invokerl_b200.algorithms import GRPO
    from invokerl_b200.policy import PolicyModel

    model, batch = setup
    tr = make_trainer(ref, SimpleNamespace(device=DEV), None)
    db = tr._batch_to_device(batch)  # the reference trainer's own device copy of the batch
    with torch.no_grad():
        lp0 = PolicyModel.from_model(model, device=DEV, dtype=torch.float32).forward(db.token_ids, db.attention_mask)
    out = {}
    for name, algo in (("ref", ref.algorithms.GRPO(clip_eps=0.2, beta=0.04)), ("ours", GRPO(clip_eps=0.2, beta=0.04))):
        lp = lp0.clone().requires_grad_(True)
        adv = algo.compute_advantages(db)
        loss, met = algo.compute_loss(lp, db, adv)
        loss.backward()
        out[name] = (float(loss.detach()), met, lp.grad.cpu(), adv.cpu())
    (lr, mr, gr, ar), (lo, mo, go, ao) = out["ref"], out["ours"]
    torch.testing.assert_close(ao, ar, rtol=1e-4, atol=1e-6)
    assert abs(lo - lr) <= 1e-4 * abs(lr) + 1e-7
    for k, v in mr.items():
        assert abs(mo[k] - v) <= 1e-4 * abs(v) + 1e-7, (k, mo[k], v)
    torch.testing.assert_close(go, gr, rtol=1e-4, atol=1e-9)
