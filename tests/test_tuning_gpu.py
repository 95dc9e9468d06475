"""Every value of every K1 launch knob (ikrl_set_tuning) against a plain fp32 PyTorch reference of
the same log-prob forward and backward.  The knobs change the kernel, tile shape, work order,
pacing and L2 hints of the tensor-core GEMMs; none may change the results beyond the tolerances
the other K1 tests use (log-probs 2e-3 absolute, gradients 1e-2 relative Frobenius)."""

import pytest
import torch

from invokerl_b200 import _native as N
from invokerl_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"

VARIANTS = (
    [{}]
    + [{"cta_pairs": 0}, {"skip_zero_rows": 0}, {"persistent": 0}, {"pace": 0}, {"pace": 3}, {"pace": 15}, {"pace": 14}, {"balance_splits": 0}]
    + [{"wide": v} for v in (0, 1, 2)]
    + [{"pace_kb": v} for v in (1, 7, 256)]
    + [{"pace_kb_long": v} for v in (16, 512)]
    + [{"split_tail": v} for v in (0, 1, 2)]
    + [{"dh_split_k": v} for v in (0, 2, 3, 16)]
    + [{"pace_lag": v} for v in (0, 2, 5)]
    + [{"l2_policy": 10 * a + b} for a in range(3) for b in range(3)]
    + [{"l2_budget_mb": v} for v in (1, 8, 200)]
)

# (rows, H, V): the 0.6B head width (wide tiles from K = 1024, 256 x 256 pair tiles for its dH),
# the 8B head width over the whole vocabulary, and a narrow head below the wide threshold.
SHAPES = [(1536, 1024, 32768), (1024, 4096, 151936), (700, 256, 5000)]


def torch_reference(h, w, t, g):
    """fp32 log-probs, dH and dW of F.linear + log-softmax gather (policy.py:173-191)."""
    logits = h.float() @ w.float().t()
    lse = torch.logsumexp(logits, dim=1)
    lp = logits.gather(1, t[:, None]).squeeze(1) - lse
    dl = -torch.softmax(logits, dim=1)
    dl.scatter_add_(1, t[:, None], torch.ones_like(t[:, None], dtype=dl.dtype))
    dl *= g[:, None]
    return lp, dl @ w.float(), dl.t() @ h.float()


def rel_fro(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp(min=1e-30))


@pytest.fixture(scope="module")
def cases():
    out = []
    for i, (n, H, V) in enumerate(SHAPES):
        gen = torch.Generator(device=DEV).manual_seed(100 + i)
        h = torch.randn(n, H, device=DEV, generator=gen).to(torch.bfloat16)
        w = (0.05 * torch.randn(V, H, device=DEV, generator=gen)).to(torch.bfloat16)
        t = torch.randint(0, V, (n,), device=DEV, generator=gen)
        g = torch.randn(n, device=DEV, generator=gen) * (torch.rand(n, device=DEV, generator=gen) < 0.5)
        out.append((h, w, t, g, torch_reference(h, w, t, g)))
    return out


@pytest.mark.parametrize("knobs", VARIANTS, ids=lambda k: ",".join(f"{a}={b}" for a, b in k.items()) or "default")
def test_knob_value_matches_fp32_reference(knobs, cases):
    before = {k: N.get_tuning(k) for k in N.TUNE}
    with N.tuning(**knobs):
        for h, w, t, g, (lp_r, dh_r, dw_r) in cases:
            lp, lse = ops.lmhead_forward_raw(h, w, t)
            dh, dw = ops.lmhead_backward_raw(h, w, t, lse, g, dw_dtype=torch.float32, chunk_rows=512)
            torch.cuda.synchronize()
            assert float((lp - lp_r).abs().max()) <= 2e-3
            assert rel_fro(dh, dh_r) <= 1e-2
            assert rel_fro(dw, dw_r) <= 1e-2
            assert float(dh[g == 0].abs().max()) == 0.0
    assert {k: N.get_tuning(k) for k in N.TUNE} == before
