"""The K1 logit cache: the forward stores per-chunk softmax numerators for the rows that may carry
a gradient, and the backward forms those rows' dlogits from them instead of recomputing the
logits.  Checked against the plain recompute path and the fp32 oracle, with rows that are cached,
rows that are active but not cached (outside the mask, or past the cache's capacity), several
backward chunks, and the autograd op's memory policy."""

import pytest
import torch

import oracle
from invokerl_b200 import _native as N
from invokerl_b200 import ops
from invokerl_b200.synthetic import lmhead_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_fro(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp(min=1e-30))


@pytest.fixture(autouse=True)
def check_device_status(monkeypatch):
    monkeypatch.setattr(ops, "_CHECK_DEVICE_STATUS", True)


@pytest.mark.parametrize("N_,H,V,chunk,cap_frac", [
    (1000, 256, 33000, 256, 1.0),      # several chunks of cached rows, then recomputed ones
    (700, 4096, 151936, None, 1.0),    # Qwen3-8B head shape, one chunk
    (3000, 1024, 151936, 512, 0.5),    # Qwen3-0.6B head width; the cache holds half the candidates
    (300, 64, 5000, None, 1.0),        # narrow head (single-K-tile pair kernel), ragged V tail
])
def test_cached_backward_matches_recompute_and_oracle(N_, H, V, chunk, cap_frac):
    li = lmhead_inputs(N_, H, V, seed=N_ + V, w_std=0.05 if H > 512 else 0.3)
    gen = torch.Generator().manual_seed(4)
    mask = torch.rand(N_, generator=gen) < 0.7          # cache candidates
    g = torch.randn(N_, generator=gen) * (torch.rand(N_, generator=gen) < 0.6)  # active rows
    t = li.targets.clone()
    t[::17] = -100                                      # ignored rows: never cached, never active
    h, w, td, gd, md = li.hidden.to(DEV), li.weight.to(DEV), t.to(DEV), g.to(DEV).float(), mask.to(DEV)
    cand = int((mask & (t != -100)).sum())
    cap = max(1, int(cand * cap_frac))
    cache = ops.LogitCache(N_, V, cap, DEV)
    lp_c, lse_c = ops.lmhead_forward_raw(h, w, td, cache, md)
    lp_p, lse_p = ops.lmhead_forward_raw(h, w, td)
    torch.cuda.synchronize()
    # the cache stores are additions to the same arithmetic: identical log-probs
    assert torch.equal(lp_c, lp_p) and torch.equal(lse_c, lse_p)
    # slots: candidates with a target, numbered in row order, up to the capacity
    want = (mask & (t != -100)).numpy()
    k, slots = 0, []
    for r in range(N_):
        slots.append(k if (want[r] and k < cap) else -1)
        k += int(want[r])
    assert cache.slot.cpu().tolist() == slots
    dh_c, dw_c = ops.lmhead_backward_raw(h, w, td, lse_c, gd, dw_dtype=torch.float32, chunk_rows=chunk, cache=cache)
    dh_p, dw_p = ops.lmhead_backward_raw(h, w, td, lse_p, gd, dw_dtype=torch.float32, chunk_rows=chunk)
    torch.cuda.synchronize()
    # the cached rows' dlogits differ from the recomputed ones by the bf16 rounding of the numerators
    assert rel_fro(dh_c, dh_p) <= 5e-3
    assert rel_fro(dw_c, dw_p) <= 5e-3
    assert float(dh_c[(gd == 0) | (td == -100)].abs().max()) == 0.0
    keep = t != -100
    lp_o, dh_o, dw_o = oracle.lmhead_logprob_grads(li.hidden[keep], li.weight, t[keep], g[keep])
    assert float((lp_c.cpu()[keep] - lp_o).abs().max()) <= 2e-3
    assert rel_fro(dh_c.cpu()[keep], dh_o) <= 1e-2
    assert rel_fro(dw_c.cpu(), dw_o) <= 1e-2


@pytest.mark.parametrize("knobs", [{"cta_pairs": 0}, {"wide": 1}, {"wide": 0}, {"skip_zero_rows": 0}])
def test_cache_under_each_kernel_choice(knobs):
    """The caching forward in the single-CTA, wide-pair and 256 x 256 pair kernels, and a backward
    that does not compact rows (the cache then goes unused): gradients as without the cache."""
    N_, H, V = 900, 512, 20000
    li = lmhead_inputs(N_, H, V, seed=21, w_std=0.1)
    gen = torch.Generator().manual_seed(3)
    g = torch.randn(N_, generator=gen) * (torch.rand(N_, generator=gen) < 0.5)
    h, w, td, gd = li.hidden.to(DEV), li.weight.to(DEV), li.targets.to(DEV), g.to(DEV)
    with N.tuning(**knobs):
        cache = ops.LogitCache(N_, V, N_, DEV)
        lp_c, lse_c = ops.lmhead_forward_raw(h, w, td, cache, None)
        lp_p, lse_p = ops.lmhead_forward_raw(h, w, td)
        dh_c, dw_c = ops.lmhead_backward_raw(h, w, td, lse_c, gd, dw_dtype=torch.float32, chunk_rows=256,
                                             cache=cache)
        dh_p, dw_p = ops.lmhead_backward_raw(h, w, td, lse_p, gd, dw_dtype=torch.float32, chunk_rows=256)
        torch.cuda.synchronize()
    assert torch.equal(lp_c, lp_p)
    assert rel_fro(dh_c, dh_p) <= 5e-3 and rel_fro(dw_c, dw_p) <= 5e-3
    _, dh_o, dw_o = oracle.lmhead_logprob_grads(li.hidden, li.weight, li.targets, g)
    assert rel_fro(dh_c.cpu(), dh_o) <= 1e-2 and rel_fro(dw_c.cpu(), dw_o) <= 1e-2


def test_every_row_cached_and_active():
    """All rows active and all cached: the backward still reorders (cached class first) and
    scatters dH back to the original rows."""
    N_, H, V = 600, 512, 8192
    li = lmhead_inputs(N_, H, V, seed=11, w_std=0.1)
    g = torch.randn(N_, generator=torch.Generator().manual_seed(2))
    h, w, td, gd = li.hidden.to(DEV), li.weight.to(DEV), li.targets.to(DEV), g.to(DEV)
    cache = ops.LogitCache(N_, V, N_, DEV)
    _, lse = ops.lmhead_forward_raw(h, w, td, cache, None)
    dh_c, dw_c = ops.lmhead_backward_raw(h, w, td, lse, gd, dw_dtype=torch.float32, chunk_rows=256, cache=cache)
    dh_p, dw_p = ops.lmhead_backward_raw(h, w, td, lse, gd, dw_dtype=torch.float32, chunk_rows=256)
    torch.cuda.synchronize()
    assert int((cache.slot >= 0).sum()) == N_
    assert rel_fro(dh_c, dh_p) <= 5e-3 and rel_fro(dw_c, dw_p) <= 5e-3


def test_autograd_op_uses_the_cache_and_matches_the_uncached_op():
    N_, H, V = 4096, 2048, 151936
    li = lmhead_inputs(N_, H, V, seed=5, w_std=0.05)
    gen = torch.Generator().manual_seed(6)
    rows = torch.rand(N_, generator=gen) < 0.5
    up = torch.randn(N_, generator=gen) * rows  # the loss weights only candidate rows
    grads = {}
    for mode in ("auto", "off"):
        prev = ops.set_logit_cache(mode)
        try:
            h = li.hidden.to(DEV).requires_grad_(True)
            w = li.weight.to(DEV).requires_grad_(True)
            lp = ops.lmhead_logprob(h, w, li.targets.to(DEV), cache_rows=rows.to(DEV))
            (lp * up.to(DEV)).sum().backward()
            torch.cuda.synchronize()
            grads[mode] = (lp.detach(), h.grad, w.grad, dict(ops.LOGIT_CACHE_STATS))
        finally:
            ops.set_logit_cache(prev["mode"])
    lp_a, dh_a, dw_a, st_a = grads["auto"]
    lp_o, dh_o, dw_o, st_o = grads["off"]
    assert st_a["rows"] == int(rows.sum()) and st_o["rows"] == 0
    assert torch.equal(lp_a, lp_o)
    assert rel_fro(dh_a, dh_o) <= 5e-3 and rel_fro(dw_a, dw_o) <= 5e-3


def test_policy_skips_narrow_heads():
    """Below H = 2048 the cache costs more than the recompute it saves; "auto" does not cache."""
    assert ops.logit_cache_rows(4096, 1024, 151936, torch.device(DEV), 4096) == 0
    assert ops.logit_cache_rows(4096, 4096, 151936, torch.device(DEV), 4096) == 4096


def test_no_gradient_no_cache():
    h = torch.randn(256, 128, device=DEV).to(torch.bfloat16)
    w = (0.1 * torch.randn(4096, 128, device=DEV)).to(torch.bfloat16)
    t = torch.randint(0, 4096, (256,), device=DEV)
    ops.LOGIT_CACHE_STATS.update(rows=-1, candidates=-1)
    with torch.no_grad():
        ops.lmhead_logprob(h, w, t)
    assert ops.LOGIT_CACHE_STATS["rows"] == -1  # the forward without a gradient never sizes a cache
