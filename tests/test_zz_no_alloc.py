"""The allocation-free LM-head forward (`ikrl_lmhead_logprob_fwd_noalloc`).

Some callers cannot allocate device memory when they need log-probs: a host application whose own
allocator owns all of the GPU's memory and forbids side allocations, or a framework whose caching
pool has already reserved the free memory.  They use this entry point: its scratch is a fixed
4 MiB array inside the library.  These tests call it through the C ABI twice in a row (different
shapes, so the second call runs on whatever the first left in the shared array) and check each
result bit for bit against the workspace-taking entry point, which runs the same kernels with the
same launch plan, and against the CPU oracle; they read the device status word of the built-in
scratch after every call, and check that a call too large for the scratch is refused before any
GPU work.

The file is named so that pytest collects it last.
"""

import pytest
import torch

import oracle
from invokerl_b200 import _native as N
from invokerl_b200.synthetic import lmhead_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


def forward_with_workspace(h, w, t):
    n, H = h.shape
    V = w.shape[0]
    logp = torch.empty(n, dtype=torch.float32, device=DEV)
    lse = torch.empty(n, dtype=torch.float32, device=DEV)
    nbytes = int(N.lib().ikrl_lmhead_fwd_workspace_bytes(n, H, V))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    N.call("ikrl_lmhead_logprob_fwd", N.ptr(h), N.ptr(w), N.ptr(t), N.i64(n), N.i32(H), N.i32(V), N.ptr(logp),
           N.ptr(lse), N.ptr(ws), N.sz(nbytes), N.stream_of(h.device))
    return logp, lse


def forward_no_alloc(h, w, t):
    n, H = h.shape
    V = w.shape[0]
    logp = torch.empty(n, dtype=torch.float32, device=DEV)
    lse = torch.empty(n, dtype=torch.float32, device=DEV)
    N.call("ikrl_lmhead_logprob_fwd_noalloc", N.ptr(h), N.ptr(w), N.ptr(t), N.i64(n), N.i32(H), N.i32(V),
           N.ptr(logp), N.ptr(lse), N.stream_of(h.device))
    return logp, lse


def no_alloc_status() -> int:
    st = N.c_int32(-1)
    N.call("ikrl_lmhead_noalloc_status", N.byref(st), N.stream_of(torch.device(DEV)))
    return int(st.value)


@pytest.mark.parametrize("shapes", [[(512, 1024, 151936), (200, 256, 5000)]])
def test_no_alloc_forward_matches_workspace_forward_twice(shapes):
    for i, (n, H, V) in enumerate(shapes):
        li = lmhead_inputs(n, H, V, seed=40 + i, w_std=0.05)
        h, w, t = li.hidden.to(DEV), li.weight.to(DEV), li.targets.to(DEV)
        lp_ref, lse_ref = forward_with_workspace(h, w, t)
        lp, lse = forward_no_alloc(h, w, t)
        torch.cuda.synchronize()
        assert no_alloc_status() == 0
        assert torch.isfinite(lp).all()
        # the same kernels, launch plan and fixed-order combine on the same inputs: bit-identical
        assert torch.equal(lp, lp_ref)
        assert torch.equal(lse, lse_ref)
        # and the oracle's fp32 log-probs within the tests' log-prob tolerance, 2e-3 absolute
        lp_o = oracle.lmhead_logprob(li.hidden, li.weight, li.targets)
        assert float((lp.cpu() - lp_o).abs().max()) <= 2e-3


def test_no_alloc_forward_rejects_rows_beyond_its_scratch():
    n, H, V = 1 << 20, 4096, 151936  # needs far more than the built-in 4 MiB
    need = int(N.lib().ikrl_lmhead_fwd_workspace_bytes(n, H, V))
    assert need > (4 << 20)
    fake = N.c_void_p(1 << 20)  # never dereferenced: the size check comes first
    with pytest.raises(N.IkrlError, match="built-in"):
        N.call("ikrl_lmhead_logprob_fwd_noalloc", fake, fake, fake, N.i64(n), N.i32(H), N.i32(V), fake, fake,
               N.c_void_p(0))
