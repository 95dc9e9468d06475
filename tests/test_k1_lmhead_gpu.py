"""K1 parity on the GPU: the fused tcgen05 LM-head log-prob forward/backward against the
reference golden vectors, the CPU oracle, and size-independent properties at full size."""

import pytest
import torch

import oracle
from helpers import load
from invokerl_b200 import _native as N
from invokerl_b200._native import tuning as launch_knobs
from invokerl_b200 import ops
from invokerl_b200.synthetic import lmhead_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def check_device_status(monkeypatch):
    # read the kernels' device status word after every call
    monkeypatch.setattr(ops, "_CHECK_DEVICE_STATUS", True)


@pytest.fixture(params=["cta_pairs", "single_cta"])
def kernel_variant(request):
    """Run a test on both K1 GEMM kernels: CTA pairs (cta_group::2) and single CTAs."""
    prev = N.lib().ikrl_lmhead_set_cta_pairs(1 if request.param == "cta_pairs" else 0)
    yield request.param
    N.lib().ikrl_lmhead_set_cta_pairs(prev)


def rel_fro(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp(min=1e-30))


def run_k1(h, w, t, g, chunk_rows=None, dw_dtype=torch.bfloat16):
    hd, wd, td = h.to(DEV), w.to(DEV), t.to(DEV)
    lp, lse = ops.lmhead_forward_raw(hd, wd, td)
    dh, dw = ops.lmhead_backward_raw(hd, wd, td, lse, g.to(DEV).float().contiguous(), dw_dtype=dw_dtype,
                                     chunk_rows=chunk_rows)
    torch.cuda.synchronize()
    return lp.cpu(), lse.cpu(), dh.cpu(), dw.cpu()


def test_golden_small(kernel_variant):
    g = load("lmhead_small")
    h = g["hidden"].reshape(-1, g["hidden"].shape[-1])
    t = g["targets"].reshape(-1)
    lp, _, dh, dw = run_k1(h, g["weight"], t, g["upstream"].reshape(-1))
    assert float((lp - g["lp_fp32"].reshape(-1)).abs().max()) <= 2e-3
    assert rel_fro(dh, g["dh_fp32"].reshape(dh.shape)) <= 1e-2
    assert rel_fro(dw, g["dw_fp32"]) <= 1e-2


def test_golden_reference_chunked_branch(kernel_variant):
    """The reference's chunk loop (B*T*V*4 >= 2 GiB) on the full vocabulary; H=32 < one K tile."""
    g = load("lmhead_chunked_seed")
    B, T, H, V = g["shape"]
    li = lmhead_inputs(B * T, H, V, seed=g["seed"], w_std=g["w_std"])
    lp, _ = ops.lmhead_forward_raw(li.hidden.to(DEV), li.weight.to(DEV), li.targets.to(DEV))
    assert float((lp.cpu() - g["lp_fp32"].reshape(-1)).abs().max()) <= 2e-3


@pytest.mark.parametrize("N,H,V,chunk", [
    (300, 128, 5000, None),        # ragged rows and vocab tail (5000 = 19*256 + 136)
    (129, 64, 1000, 64),           # several chunks, tail chunk of 1 row
    (600, 256, 33000, 256),        # 3 chunks with a ragged last one
    (256, 1024, 151936, None),     # Qwen3-0.6B head shape
    (160, 4096, 151936, 128),      # Qwen3-8B head shape, 2 chunks
    (40, 200, 777, None),          # H not a multiple of 64, V odd
])
def test_against_oracle(N, H, V, chunk, kernel_variant):
    li = lmhead_inputs(N, H, V, seed=N + H + V, w_std=0.05 if H > 512 else 0.3)
    gen = torch.Generator().manual_seed(1)
    g = torch.randn(N, generator=gen) * torch.bernoulli(torch.full((N,), 0.7), generator=gen)
    lp, lse, dh, dw = run_k1(li.hidden, li.weight, li.targets, g, chunk_rows=chunk)
    lp_o, dh_o, dw_o = oracle.lmhead_logprob_grads(li.hidden, li.weight, li.targets, g)
    assert float((lp - lp_o).abs().max()) <= 2e-3
    assert rel_fro(dh, dh_o) <= 1e-2
    assert rel_fro(dw, dw_o) <= 1e-2
    # rows with zero upstream have exactly zero hidden gradient
    z = g == 0
    if z.any():
        assert float(dh[z].abs().max()) == 0.0


def test_fp32_dweight_accumulates(kernel_variant):
    N, H, V = 200, 128, 3000
    li = lmhead_inputs(N, H, V, seed=3, w_std=0.3)
    g = torch.randn(N, generator=torch.Generator().manual_seed(2))
    hd, wd, td = li.hidden.to(DEV), li.weight.to(DEV), li.targets.to(DEV)
    _, lse = ops.lmhead_forward_raw(hd, wd, td)
    base = torch.randn(V, H, device=DEV)
    acc = base.clone()
    ops.lmhead_backward_raw(hd, wd, td, lse, g.to(DEV), want_dh=False, dweight_out=acc, chunk_rows=128)
    _, _, dw_o = oracle.lmhead_logprob_grads(li.hidden, li.weight, li.targets, g)
    assert rel_fro((acc - base).cpu(), dw_o) <= 1e-2


def test_ignored_rows_and_autograd_function():
    N, H, V = 96, 64, 2048
    li = lmhead_inputs(N, H, V, seed=5, w_std=0.3)
    t = li.targets.clone()
    t[::7] = -100
    h = li.hidden.to(DEV).requires_grad_(True)
    w = li.weight.to(DEV).requires_grad_(True)
    lp = ops.lmhead_logprob(h, w, t.to(DEV))
    up = torch.randn(N, generator=torch.Generator().manual_seed(4))
    (lp * up.to(DEV)).sum().backward()
    keep = t != -100
    assert (lp.detach().cpu()[~keep] == 0).all()
    lp_o, dh_o, dw_o = oracle.lmhead_logprob_grads(li.hidden[keep], li.weight, t[keep], up[keep])
    assert float((lp.detach().cpu()[keep] - lp_o).abs().max()) <= 2e-3
    assert float(h.grad.cpu()[~keep].abs().max()) == 0.0
    assert rel_fro(h.grad.cpu()[keep], dh_o) <= 1e-2
    assert rel_fro(w.grad.cpu(), dw_o) <= 1e-2


@pytest.mark.parametrize("N,H", [(131072, 1024), (65536, 4096)])
def test_full_size_properties(N, H, kernel_variant):
    """Config-3 size (and half of config 4's rows): log-probs of sampled rows against the oracle;
    dH of sampled rows; dW on sampled vocab rows from the kernel's own lse; sum_v dW[v] = 0."""
    V = 151936
    gen = torch.Generator(device=DEV).manual_seed(7)
    h = torch.randn(N, H, device=DEV, generator=gen).to(torch.bfloat16)
    w = (0.02 * torch.randn(V, H, device=DEV, generator=gen)).to(torch.bfloat16)
    t = torch.randint(0, V, (N,), device=DEV, generator=gen)
    g = torch.randn(N, device=DEV, generator=gen)
    lp, lse = ops.lmhead_forward_raw(h, w, t)
    dh, dw = ops.lmhead_backward_raw(h, w, t, lse, g, dw_dtype=torch.float32)
    torch.cuda.synchronize()
    rows = torch.randint(0, N, (48,), generator=torch.Generator().manual_seed(0))
    hs, ws, ts, gs = h[rows].cpu(), w.cpu(), t[rows].cpu(), g[rows].cpu()
    lp_o, dh_o, _ = oracle.lmhead_logprob_grads(hs, ws, ts, gs)
    assert float((lp[rows].cpu() - lp_o).abs().max()) <= 2e-3
    lse_o = torch.logsumexp(hs.float() @ ws.float().t(), dim=1)
    assert float((lse[rows].cpu() - lse_o).abs().max()) <= 2e-3
    assert rel_fro(dh[rows].cpu(), dh_o) <= 1e-2
    # dW on a vocab subset: sum_n g_n ([t_n = v] - exp(h_n.W_v - lse_n)) h_n, from the kernel's lse
    vs = torch.randint(0, V, (16,), generator=torch.Generator().manual_seed(1))
    hf = h.float()
    p = torch.exp(hf @ w[vs.to(DEV)].float().t() - lse[:, None])  # [N, 16] on the GPU (fp32 torch)
    onehot = (t[:, None] == vs.to(DEV)[None, :]).float()
    dw_sub = ((onehot - p) * g[:, None]).t() @ hf
    assert rel_fro(dw[vs.to(DEV)], dw_sub) <= 1e-2
    colsum = dw.sum(dim=0)
    assert float(colsum.norm() / dw.norm()) <= 1e-2


def _bwd(h, w, t, lse, g, skip: bool, **kw):
    with N.tuning(skip_zero_rows=1 if skip else 0):
        out = ops.lmhead_backward_raw(h, w, t, lse, g, **kw)
        torch.cuda.synchronize()
        return out


@pytest.mark.parametrize("N,H,V,chunk,frac", [
    (1000, 256, 33000, 256, 0.4),      # several chunks of compacted rows
    (700, 4096, 151936, None, 0.5),    # Qwen3-8B head shape, one chunk
    (2500, 64, 5000, 512, 0.02),       # very few active rows (fewer than one chunk)
])
def test_zero_gradient_rows_are_skipped_exactly(N, H, V, chunk, frac, kernel_variant):
    """Rows with zero upstream gradient (masked tokens) and ignore_index rows are left out of the
    backward GEMMs: dH is identical to the dense computation when both split the vocabulary
    reduction of dH into the same K ranges (the automatic choice depends on the row count, so
    there the two agree to bf16 rounding), dW equal up to fp32 summation order."""
    li = lmhead_inputs(N, H, V, seed=N + V, w_std=0.05 if H > 512 else 0.3)
    gen = torch.Generator().manual_seed(9)
    g = torch.randn(N, generator=gen) * torch.bernoulli(torch.full((N,), frac), generator=gen)
    t = li.targets.clone()
    t[torch.bernoulli(torch.full((N,), 0.05), generator=gen).bool()] = -100
    hd, wd, td, gd = li.hidden.to(DEV), li.weight.to(DEV), t.to(DEV), g.to(DEV)
    _, lse = ops.lmhead_forward_raw(hd, wd, td)
    for ks in (0, 3):
        with launch_knobs(dh_split_k=ks):
            dh_s, _ = _bwd(hd, wd, td, lse, gd, True, dw_dtype=torch.float32, chunk_rows=chunk)
            dh_d, _ = _bwd(hd, wd, td, lse, gd, False, dw_dtype=torch.float32, chunk_rows=chunk)
        assert torch.equal(dh_s, dh_d)
    dh_s, dw_s = _bwd(hd, wd, td, lse, gd, True, dw_dtype=torch.float32, chunk_rows=chunk)
    dh_d, dw_d = _bwd(hd, wd, td, lse, gd, False, dw_dtype=torch.float32, chunk_rows=chunk)
    assert rel_fro(dh_s, dh_d) <= 4e-3
    torch.testing.assert_close(dw_s, dw_d, rtol=1e-4, atol=1e-6)
    dead = (g == 0) | (t == -100)
    assert float(dh_s.cpu()[dead].abs().max()) == 0.0
    keep = t != -100
    _, dh_o, dw_o = oracle.lmhead_logprob_grads(li.hidden[keep], li.weight, t[keep], g[keep])
    assert rel_fro(dh_s.cpu()[keep], dh_o) <= 1e-2
    assert rel_fro(dw_s.cpu(), dw_o) <= 1e-2
    # bf16 dW through the fp32 workspace when the compacted rows span several chunks
    _, dw_b = _bwd(hd, wd, td, lse, gd, True, want_dh=False, dw_dtype=torch.bfloat16, chunk_rows=chunk)
    assert rel_fro(dw_b.cpu(), dw_o) <= 1e-2


def test_all_rows_zero_gradient():
    N, H, V = 300, 128, 3000
    li = lmhead_inputs(N, H, V, seed=11, w_std=0.3)
    hd, wd, td = li.hidden.to(DEV), li.weight.to(DEV), li.targets.to(DEV)
    _, lse = ops.lmhead_forward_raw(hd, wd, td)
    g = torch.zeros(N, device=DEV)
    dh, dw = _bwd(hd, wd, td, lse, g, True, dw_dtype=torch.bfloat16)
    assert float(dh.abs().max()) == 0.0 and float(dw.abs().max()) == 0.0
    base = torch.randn(V, H, device=DEV)
    acc = base.clone()
    _bwd(hd, wd, td, lse, g, True, want_dh=False, dweight_out=acc)
    assert torch.equal(acc, base)


def test_forward_and_backward_capture_into_a_cuda_graph(monkeypatch):
    """Both K1 calls can be captured into a CUDA graph: inside a capture the backward runs all
    rows (no host read of the active count) and the replay equals the eager results.  dH is split
    into a fixed number of K ranges, so the eager call (on the compacted rows) and the captured one
    (on all rows) sum the same partials."""
    monkeypatch.setattr(ops, "_CHECK_DEVICE_STATUS", False)  # the status read synchronises
    with launch_knobs(dh_split_k=4):
        _capture_and_compare()


def _capture_and_compare():
    N, H, V = 512, 4096, 20000
    li = lmhead_inputs(N, H, V, seed=21, w_std=0.05)
    h, w, t = li.hidden.to(DEV), li.weight.to(DEV), li.targets.to(DEV)
    g = (torch.randn(N, generator=torch.Generator().manual_seed(22)) * (torch.arange(N) % 2)).to(DEV)
    lp_e, lse_e = ops.lmhead_forward_raw(h, w, t)
    dh_e, dw_e = ops.lmhead_backward_raw(h, w, t, lse_e, g, dw_dtype=torch.float32)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):  # warm-up on the capture stream
        ops.lmhead_forward_raw(h, w, t)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        lp_c, lse_c = ops.lmhead_forward_raw(h, w, t)
        dh_c, dw_c = ops.lmhead_backward_raw(h, w, t, lse_c, g, dw_dtype=torch.float32)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(lp_c, lp_e) and torch.equal(lse_c, lse_e)
    assert torch.equal(dh_c, dh_e)
    torch.testing.assert_close(dw_c, dw_e, rtol=1e-4, atol=1e-6)


def test_empty_batch():
    """No rows: empty outputs, a zero weight gradient (unchanged when accumulating), status 0."""
    H, V = 128, 3000
    w = lmhead_inputs(1, H, V, seed=5, w_std=0.3).weight.to(DEV)
    h = torch.empty(0, H, dtype=torch.bfloat16, device=DEV)
    t = torch.empty(0, dtype=torch.int64, device=DEV)
    lp, lse = ops.lmhead_forward_raw(h, w, t)
    assert lp.shape == (0,) and lse.shape == (0,)
    g = torch.empty(0, device=DEV)
    for dw_dtype in (torch.bfloat16, torch.float32):
        dh, dw = ops.lmhead_backward_raw(h, w, t, lse, g, dw_dtype=dw_dtype)
        assert dh.shape == (0, H) and dw.dtype == dw_dtype and float(dw.abs().max()) == 0.0
    base = torch.randn(V, H, device=DEV)
    acc = base.clone()
    ops.lmhead_backward_raw(h, w, t, lse, g, want_dh=False, dweight_out=acc)
    assert torch.equal(acc, base)
    hr = h.requires_grad_(True)
    wr = w.float().requires_grad_(True)
    out = ops.lmhead_logprob(hr, wr, t)
    out.sum().backward()
    assert out.shape == (0,) and float(wr.grad.abs().max()) == 0.0
