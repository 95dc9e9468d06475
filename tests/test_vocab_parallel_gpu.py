"""Vocab-parallel LM head on one GPU: the shards of W run one after another and the exchange is
done in-process (stack instead of all-gather, sum instead of all-reduce).  Log-probs, lse, dH
and dW must equal the unsharded fused kernel and the oracle."""

import pytest
import torch

import oracle
from invokerl_b200 import ops
from invokerl_b200.synthetic import lmhead_inputs
from invokerl_b200.vocab_parallel import (combine, lmhead_logprob_vocab_parallel, shard_backward_raw, shard_bounds,
                                          shard_forward_raw)

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def check_device_status(monkeypatch):
    monkeypatch.setattr(ops, "_CHECK_DEVICE_STATUS", True)


def rel_fro(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp(min=1e-30))


@pytest.mark.parametrize("N,H,V,P", [(300, 128, 5000, 2), (257, 256, 33000, 3), (200, 4096, 151936, 8)])
def test_emulated_shards_match_unsharded(N, H, V, P):
    li = lmhead_inputs(N, H, V, seed=N + P, w_std=0.05 if H > 512 else 0.3)
    gen = torch.Generator().manual_seed(5)
    t = li.targets.clone()
    t[torch.bernoulli(torch.full((N,), 0.05), generator=gen).bool()] = -100
    g = torch.randn(N, generator=gen) * torch.bernoulli(torch.full((N,), 0.6), generator=gen)
    h, w, td, gd = li.hidden.to(DEV), li.weight.to(DEV), t.to(DEV), g.to(DEV)
    parts, bounds = [], []
    for r in range(P):
        s, e = shard_bounds(V, P, r)
        bounds.append((s, e))
        tl, ls = shard_forward_raw(h, w[s:e].contiguous(), td, s)
        parts.append(torch.stack([tl, ls]))
    logp, lse = combine(torch.stack(parts), td, V)
    lp_u, lse_u = ops.lmhead_forward_raw(h, w, td)
    keep = t != -100
    assert torch.equal(logp.cpu()[~keep.cpu()], lp_u.cpu()[~keep.cpu()])
    assert float((logp - lp_u).abs()[keep.to(DEV)].max()) <= 1e-4
    assert float((lse - lse_u).abs().max()) <= 1e-4
    dh = torch.zeros(N, H, dtype=torch.float32, device=DEV)
    dws = []
    for r, (s, e) in enumerate(bounds):
        dh_r, dw_r = shard_backward_raw(h, w[s:e].contiguous(), td, lse, gd, s, dw_dtype=torch.float32)
        dh += dh_r.float()
        dws.append(dw_r)
    dw = torch.cat(dws)
    _, dh_o, dw_o = oracle.lmhead_logprob_grads(li.hidden[keep], li.weight, t[keep], g[keep])
    assert rel_fro(dh.cpu()[keep], dh_o) <= 1e-2
    assert float(dh.cpu()[~keep].abs().max()) == 0.0
    assert rel_fro(dw.cpu(), dw_o) <= 1e-2
    dh_u, dw_u = ops.lmhead_backward_raw(h, w, td, lse_u, gd, dw_dtype=torch.float32)
    # dH: the unsharded result is one bf16 rounding of the sum, the sharded one a sum of P bf16
    # terms; dW: the shards' dS uses the merged lse, so a few bf16 dS values round the other way
    assert rel_fro(dh, dh_u) <= 1e-2
    assert rel_fro(dw, dw_u) <= 1e-3


def test_single_rank_autograd_equals_fused_head():
    N, H, V = 192, 64, 3000
    li = lmhead_inputs(N, H, V, seed=9, w_std=0.3)
    up = torch.randn(N, generator=torch.Generator().manual_seed(3)).to(DEV)
    h1 = li.hidden.to(DEV).requires_grad_(True)
    w1 = li.weight.to(DEV).requires_grad_(True)
    lp1 = lmhead_logprob_vocab_parallel(h1, w1, li.targets.to(DEV), 0, V)
    (lp1 * up).sum().backward()
    h2 = li.hidden.to(DEV).requires_grad_(True)
    w2 = li.weight.to(DEV).requires_grad_(True)
    lp2 = ops.lmhead_logprob(h2, w2, li.targets.to(DEV))
    (lp2 * up).sum().backward()
    assert float((lp1 - lp2).abs().max()) <= 1e-5
    assert rel_fro(h1.grad, h2.grad) <= 1e-3
    assert rel_fro(w1.grad, w2.grad) <= 1e-3
