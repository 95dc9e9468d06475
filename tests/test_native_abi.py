"""The C-ABI library builds, loads without a GPU, and exports every declared symbol."""

import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> list[str]:
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        names += re.findall(r"IKRL_API\s+[\w\s\*]+?\b(ikrl_\w+)\s*\(", h.read_text())
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from invokerl_b200.csrc.build import build

    build()
    from invokerl_b200 import _native

    return _native.lib()


def test_header_declares_symbols():
    names = declared_symbols()
    assert len(names) >= 18
    assert "ikrl_clip_loss_fwd" in names and "ikrl_logits_logprob_fwd" in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_every_declared_symbol_has_a_python_signature(lib):
    from invokerl_b200 import _native

    missing = [n for n in declared_symbols() if n not in _native.exported_names()]
    assert not missing, missing


def test_abi_version_and_error_string(lib):
    assert lib.ikrl_abi_version() >= 1
    assert lib.ikrl_last_error() == b""


def test_argument_errors_need_no_gpu(lib):
    """Validation happens on the host before any CUDA call and sets the error string."""
    from invokerl_b200 import _native as N

    with pytest.raises(N.IkrlError, match="group_size"):
        N.call("ikrl_group_advantages", None, None, None, N.i32(6), N.i32(4), N.i32(4), N.i32(0),
               N.f32(0), None, None, None)
    with pytest.raises(N.IkrlError, match="workspace"):
        N.call("ikrl_masked_moments", N.c_void_p(16), N.c_void_p(16), N.i64(10), N.c_void_p(16), None,
               N.sz(0), None)
    p = N.c_void_p(256)
    with pytest.raises(N.IkrlError, match="multiple of 8"):  # hidden rows must be 16-byte aligned
        N.call("ikrl_lmhead_logprob_fwd", p, p, p, N.i64(4), N.i32(12), N.i32(100), p, p, p, N.sz(1 << 20), None)
    with pytest.raises(N.IkrlError, match="bad sizes"):
        N.call("ikrl_lmhead_logprob_fwd", p, p, p, N.i64(-1), N.i32(64), N.i32(100), p, p, p, N.sz(1 << 20), None)
    with pytest.raises(N.IkrlError, match="bf16 dweight"):  # accumulation needs an fp32 dW
        N.call("ikrl_lmhead_logprob_bwd", p, p, p, p, p, N.i64(4), N.i32(64), N.i32(100), N.i64(0), p, p,
               N.i32(N.IKRL_DTYPE_BF16), N.i32(1), p, N.sz(1 << 20), None)


def test_cpu_tensors_are_rejected():
    import torch

    from invokerl_b200 import ops

    with pytest.raises(RuntimeError, match="CUDA"):
        ops.mask_count(torch.ones(4, dtype=torch.bool))


def test_product_package_never_reaches_the_oracle():
    """The oracle is the checker only: no module of the package imports or names it."""
    pkg = ROOT / "invokerl_b200"
    offenders = []
    for f in sorted(pkg.rglob("*.py")):
        text = f.read_text()
        if re.search(r"^\s*(import oracle|from oracle\b)", text, re.M) or "oracle." in text:
            offenders.append(str(f.relative_to(ROOT)))
    assert not offenders, offenders


def test_importing_the_package_loads_no_oracle():
    import subprocess
    import sys

    code = ("import sys, invokerl_b200, invokerl_b200.ops, invokerl_b200.policy, invokerl_b200.algorithms, "
            "invokerl_b200.vocab_parallel, invokerl_b200.rollout, invokerl_b200.distributed; "
            "print(any(m == 'oracle' or m.startswith('oracle.') for m in sys.modules))")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "False"


def _plan(gemm, rows, H, V=151936, nsm=148):
    import ctypes

    from invokerl_b200 import _native as N

    out = (ctypes.c_int32 * 4)()
    N.call("ikrl_lmhead_plan", N.i32(gemm), N.i64(rows), N.i32(H), N.i32(V), N.i32(nsm), out)
    return tuple(out)


@pytest.mark.parametrize("gemm,rows,H,want", [
    # (kernel, column tiles, tiles per unit, units per row pair); kernel 2 = wide pairs 256 x 512
    (0, 524288, 4096, (2, 297, 75, 4)),   # 8B forward: the L2 rule's 4 vocabulary splits
    (1, 28160, 4096, (2, 297, 75, 4)),    # 8B full dS chunk: 440 units on 74 pairs, kept
    (1, 8700, 4096, (2, 297, 23, 13)),    # 8B last chunk: 5 splits would run 3 rounds where the mean is 2.3
    (1, 3456, 4096, (2, 297, 20, 15)),    # 14 m-pairs: 11 splits -> 15
    (3, 28160, 4096, (2, 8, 1, 8)),       # 8B dH stays wide
    (0, 131072, 1024, (2, 297, 149, 2)),  # 0.6B forward: wide from K = 1024
    (1, 10092, 1024, (2, 297, 33, 9)),    # 0.6B dS: 4 splits -> 9
    (3, 10092, 1024, (1, 4, 1, 4)),       # 0.6B dH undivided: 256 x 256 pairs (80 wide units would run 2 rounds)
    (4, 10092, 1024, (12, 0, 0, 0)),      # ... and split: 12 K ranges, 960 units in 13 rounds
    (4, 3456, 4096, (7, 0, 0, 0)),        # 14 row pairs x 8: 7 ranges (the partials cap the count at 9)
    (4, 28160, 4096, (1, 0, 0, 0)),       # 8B full chunk: 880 units, no split
    (4, 8700, 4096, (1, 0, 0, 0)),        # 8B last chunk: 272 units, no split
    (1, 256, 64, (1, 594, 3, 198)),       # K = 64: 256 x 256 pairs
])
def test_lmhead_launch_plan(lib, gemm, rows, H, want):
    assert _plan(gemm, rows, H) == want


def test_lmhead_launch_plan_balance_off(lib):
    from invokerl_b200 import _native as N

    with N.tuning(balance_splits=0):
        assert _plan(1, 8700, 4096) == (2, 297, 60, 5)
        assert _plan(3, 10092, 1024) == (2, 2, 1, 2)
    assert _plan(1, 8700, 4096) == (2, 297, 23, 13)


def test_lmhead_launch_plan_follows_the_knobs(lib):
    from invokerl_b200 import _native as N

    with N.tuning(cta_pairs=0):
        assert _plan(0, 524288, 4096)[0] == 0
    with N.tuning(wide=0):
        assert _plan(0, 524288, 4096)[0] == 1
    with N.tuning(wide=2):  # the K >= 1024 rule without the dH balance choice
        assert _plan(3, 10092, 1024) == (2, 2, 1, 2)
    with N.tuning(l2_budget_mb=8):  # less L2 for resident rows -> more vocabulary splits
        assert _plan(0, 524288, 4096)[3] > 4
    with N.tuning(dh_split_k=0):
        assert _plan(4, 10092, 1024)[0] == 1
    with N.tuning(dh_split_k=3):  # forced, wherever the partials fit
        assert _plan(4, 28160, 4096)[0] == 1 and _plan(4, 3456, 4096)[0] == 3
    with N.tuning(wide=0):
        assert _plan(4, 10092, 1024)[0] == 1


def test_tuning_knobs_range_checks_and_defaults(lib):
    """ikrl_set_tuning validates on the host; IKRL_TUNE_DEFAULT restores the shipped default; the
    library reads no environment variable."""
    from invokerl_b200 import _native as N

    defaults = {"cta_pairs": 1, "skip_zero_rows": 1, "wide": -1, "persistent": 1, "pace": -1, "pace_kb": 128,
                "pace_lag": 1, "balance_splits": 1, "l2_policy": -1, "l2_budget_mb": 0, "loss_kernel": 1,
                "pace_kb_long": 128, "split_tail": 4, "dh_split_k": -1}
    assert {k: N.get_tuning(k) for k in N.TUNE} == defaults
    prev = N.set_tuning("pace_kb", 7)
    assert prev == 128 and N.get_tuning("pace_kb") == 7
    N.set_tuning("pace_kb", None)
    assert N.get_tuning("pace_kb") == 128
    for knob, bad in [("l2_policy", 13), ("l2_policy", 30), ("pace_kb", 0), ("wide", 3), ("loss_kernel", 3)]:
        with pytest.raises(N.IkrlError, match="ikrl_set_tuning"):
            N.set_tuning(knob, bad)
    assert {k: N.get_tuning(k) for k in N.TUNE} == defaults
    with pytest.raises(N.IkrlError, match="unknown knob"):
        N.call("ikrl_set_tuning", N.i32(99), N.i64(0), None)
    src = "".join(p.read_text() for p in sorted((ROOT / "invokerl_b200" / "csrc").glob("*.cu")))
    assert "getenv" not in src


def test_no_alloc_limits_match_the_documented_row_counts(lib):
    """The allocation-free forward's 4 MiB scratch holds the forward workspace of up to 31,772 rows
    at H = 4096 and 61,672 at H = 1024 (V = 151936), the limits its documentation states."""
    w = lib.ikrl_lmhead_fwd_workspace_bytes
    for H, rows in [(4096, 31772), (1024, 61672)]:
        assert w(rows, H, 151936) <= 4 << 20 < w(rows + 1, H, 151936)


def test_lmhead_launch_plan_rejects_bad_arguments(lib):
    from invokerl_b200 import _native as N

    with pytest.raises(N.IkrlError, match="gemm"):
        _plan(5, 100, 64)
    with pytest.raises(N.IkrlError, match="bad arguments"):
        _plan(0, 0, 64)


def test_logit_cache_layout_and_argument_checks(lib):
    from invokerl_b200 import _native as N

    q, m = N.c_int64(0), N.c_int64(0)
    N.call("ikrl_lmhead_cache_row_elems", N.i32(151936), N.byref(q), N.byref(m))
    assert (q.value, m.value) == (151936, 4748)
    N.call("ikrl_lmhead_cache_row_elems", N.i32(5000), N.byref(q), N.byref(m))
    assert (q.value, m.value) == (5056, 157)
    assert lib.ikrl_lmhead_cache_fwd_workspace_bytes(524288, 4096, 151936) > lib.ikrl_lmhead_fwd_workspace_bytes(
        524288, 4096, 151936)
    p = N.c_void_p(256)
    with pytest.raises(N.IkrlError, match="multiple of 8"):
        N.call("ikrl_lmhead_logprob_fwd_cached", p, p, p, N.i64(4), N.i32(64), N.i32(1001), p, p, None, N.i64(4),
               p, p, p, p, N.sz(1 << 20), None)
    with pytest.raises(N.IkrlError, match="null cache"):
        N.call("ikrl_lmhead_logprob_bwd_cached", p, p, p, p, p, N.i64(4), N.i32(64), N.i32(1000), N.i64(0), p, p,
               N.i32(N.IKRL_DTYPE_F32), N.i32(0), None, None, None, p, N.sz(1 << 20), None)
