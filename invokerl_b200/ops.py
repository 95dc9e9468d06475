"""PyTorch-facing ops over the C ABI: plain functions for the advantage kernels and
``torch.autograd.Function`` s for the losses and the log-prob kernels.

Every op checks that its tensors are on a CUDA device and calls the native library on the
current stream; nothing here computes on the CPU or falls back to ATen for the hot-path math.
"""

from __future__ import annotations

import torch

from . import _native as N
from ._native import call, f32, i32, i64, ptr, sz

# ---------------------------------------------------------------------------------------------
# Advantages (invokerl/algorithms/base.py:86-110, grpo.py:46-80, dapo.py:55-88, ppo.py:65-106)
# ---------------------------------------------------------------------------------------------


def mask_count(mask: torch.Tensor) -> torch.Tensor:
    """Number of True entries of `mask` as an int64 device tensor of shape [1] (no host sync)."""
    dev = N.require_cuda(mask)
    m = N.as_mask(mask)
    out = torch.empty(1, dtype=torch.int64, device=dev)
    call("ikrl_mask_count", ptr(m), i64(m.numel()), ptr(out), N.stream_of(dev))
    return out


def broadcast_advantages(rewards: torch.Tensor, response_mask: torch.Tensor) -> torch.Tensor:
    """rewards[b] * mask[b,t] (base.py:108-110)."""
    dev = N.require_cuda(rewards, response_mask)
    B, T = response_mask.shape
    r = rewards.contiguous().float()
    m = N.as_mask(response_mask)
    out = torch.empty(B, T, dtype=torch.float32, device=dev)
    call("ikrl_broadcast_advantages", ptr(r), ptr(m), i32(B), i32(T), ptr(out), N.stream_of(dev))
    return out


def group_advantages(
    rewards: torch.Tensor,
    response_mask: torch.Tensor,
    group_size: int,
    filter_zero_var: bool = False,
    truncated: torch.Tensor | None = None,
    overlong_penalty: float = 0.0,
    row_adv: torch.Tensor | None = None,
) -> torch.Tensor:
    """Group-normalised advantages broadcast over the response mask (grpo.py:72-80;
    with filter_zero_var / truncated: dapo.py:61-88)."""
    dev = N.require_cuda(rewards, response_mask, truncated)
    B, T = response_mask.shape
    if rewards.numel() != B:
        raise ValueError(f"rewards has {rewards.numel()} entries, expected B={B}")
    r = rewards.contiguous().float()
    m = N.as_mask(response_mask)
    tr = None if truncated is None else N.as_mask(truncated)
    out = torch.empty(B, T, dtype=torch.float32, device=dev)
    call(
        "ikrl_group_advantages", ptr(r), ptr(m), ptr(tr), i32(B), i32(T), i32(group_size),
        i32(1 if filter_zero_var else 0), f32(overlong_penalty), ptr(out), ptr(row_adv),
        N.stream_of(dev),
    )
    return out


def token_group_advantages(token_rewards: torch.Tensor, response_mask: torch.Tensor, group_size: int) -> torch.Tensor:
    """Per-(group, position) normalisation of token rewards (grpo.py:62-70)."""
    dev = N.require_cuda(token_rewards, response_mask)
    B, T = response_mask.shape
    tr = token_rewards.contiguous().float()
    m = N.as_mask(response_mask)
    out = torch.empty(B, T, dtype=torch.float32, device=dev)
    call("ikrl_token_group_advantages", ptr(tr), ptr(m), i32(B), i32(T), i32(group_size), ptr(out),
         N.stream_of(dev))
    return out


def gae_advantages(
    rewards: torch.Tensor | None,
    token_rewards: torch.Tensor | None,
    values: torch.Tensor,
    response_mask: torch.Tensor,
    gamma: float,
    lam: float,
) -> torch.Tensor:
    """PPO GAE reverse scan (ppo.py:80-106), one block per row."""
    dev = N.require_cuda(values, response_mask, rewards, token_rewards)
    B, T = response_mask.shape
    v = values.contiguous().float()
    m = N.as_mask(response_mask)
    rb = None if rewards is None else rewards.contiguous().float()
    rt = None if token_rewards is None else token_rewards.contiguous().float()
    out = torch.empty(B, T, dtype=torch.float32, device=dev)
    call("ikrl_gae_advantages", ptr(rb), ptr(rt), ptr(v), ptr(m), i32(B), i32(T), f32(gamma), f32(lam),
         ptr(out), N.stream_of(dev))
    return out


def masked_moments(x: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """[mean, unbiased std, count, enabled] of x over mask (ppo.py:123-127)."""
    dev = N.require_cuda(x, mask)
    xx = x.contiguous().float()
    m = N.as_mask(mask)
    n = xx.numel()
    out = torch.empty(4, dtype=torch.float32, device=dev)
    nbytes = int(N.lib().ikrl_masked_moments_workspace_bytes(n))
    ws = N.workspace(dev, nbytes)
    call("ikrl_masked_moments", ptr(xx), ptr(m), i64(n), ptr(out), ptr(ws), sz(ws.numel()), N.stream_of(dev))
    return out


# ---------------------------------------------------------------------------------------------
# Clipped-ratio loss (grpo.py:84-143, dapo.py:90-150, ppo.py:108-184)
# ---------------------------------------------------------------------------------------------


def make_loss_params(
    family: int,
    ratio_lo: float,
    ratio_hi: float,
    clip_metric_eps: float,
    beta: float,
    kl_type: str | int = "schulman",
    entropy_coef: float = 0.0,
    vf_coef: float = 0.0,
    vf_clip_eps: float = 0.0,
) -> N.LossParams:
    if isinstance(kl_type, str):
        kl = N.IKRL_KL_SCHULMAN if kl_type == "schulman" else N.IKRL_KL_SIMPLE
    else:
        kl = int(kl_type)
    return N.LossParams(family, ratio_lo, ratio_hi, clip_metric_eps, beta, kl, entropy_coef, vf_coef,
                        vf_clip_eps)


def _clip_loss_launch(new_lp, old_lp, ref_lp, adv, mask_u8, rewards, G, ntok, whiten, values, old_values,
                      params, want_dlp, want_dvalues):
    dev = new_lp.device
    B, T = new_lp.shape
    dlp = torch.empty_like(new_lp) if want_dlp else None
    dvalues = torch.empty(B, T, dtype=torch.float32, device=dev) if want_dvalues else None
    sums = torch.empty(N.LOSS_NSUMS, dtype=torch.float64, device=dev)
    nbytes = int(N.lib().ikrl_clip_loss_workspace_bytes(B * T))
    ws = N.workspace(dev, nbytes)
    call(
        "ikrl_clip_loss_fwd", ptr(new_lp), i32(N.dtype_code(new_lp)), ptr(old_lp), ptr(ref_lp), ptr(adv),
        ptr(mask_u8), ptr(rewards), i32(B), i32(T), i32(G), ptr(ntok), ptr(whiten), ptr(values),
        ptr(old_values), params, ptr(dlp), ptr(dvalues), ptr(sums), ptr(ws), sz(ws.numel()),
        N.stream_of(dev),
    )
    return dlp, dvalues, sums


def clip_loss_finalize(sums: torch.Tensor, ntok: torch.Tensor, params: N.LossParams):
    dev = sums.device
    loss = torch.empty((), dtype=torch.float32, device=dev)
    metrics = torch.empty(N.LOSS_NMETRICS, dtype=torch.float32, device=dev)
    call("ikrl_clip_loss_finalize", ptr(sums), ptr(ntok), params, ptr(loss), ptr(metrics), N.stream_of(dev))
    return loss, metrics


def _scale(g_tensor: torch.Tensor, upstream: torch.Tensor) -> None:
    s = upstream.detach().reshape(1).to(torch.float32).contiguous()
    call("ikrl_scale_grad", ptr(g_tensor), i32(N.dtype_code(g_tensor)), i64(g_tensor.numel()), ptr(s),
         N.stream_of(g_tensor.device))


class ClipRatioLoss(torch.autograd.Function):
    """Loss value of one rank's rows; d loss / d new_lp is written by the forward pass and scaled
    by the upstream gradient in backward (skipped on the device when the upstream is 1)."""

    @staticmethod
    def forward(ctx, new_lp, values, old_lp, ref_lp, adv, mask_u8, rewards, G, ntok, whiten, old_values,
                params):
        want_dlp = new_lp.requires_grad
        want_dv = values is not None and values.requires_grad
        dlp, dvalues, sums = _clip_loss_launch(
            new_lp.detach(), old_lp, ref_lp, adv, mask_u8, rewards, G, ntok, whiten,
            None if values is None else values.detach(), old_values, params, want_dlp, want_dv,
        )
        loss, _ = clip_loss_finalize(sums, ntok, params)
        ctx.dlp = dlp
        ctx.dvalues = dvalues
        ctx.n_bwd = 0
        ctx.replay = (new_lp.detach(), None if values is None else values.detach(), old_lp, ref_lp, adv, mask_u8,
                      rewards, G, ntok, whiten, old_values, params, want_dlp, want_dv)
        ctx.mark_non_differentiable(sums)
        return loss, sums

    @staticmethod
    def backward(ctx, g_loss, g_sums):
        if g_loss is None:
            return (None,) * 12
        dlp, dvalues = ctx.dlp, ctx.dvalues
        if ctx.n_bwd > 0:  # retain_graph: the saved gradient was scaled in place; recompute it
            (nl, vals, old, ref, adv, m, r, G, ntok, wh, ov, params, wd, wv) = ctx.replay
            dlp, dvalues, _ = _clip_loss_launch(nl, old, ref, adv, m, r, G, ntok, wh, vals, ov, params, wd, wv)
        ctx.n_bwd += 1
        if dlp is not None:
            _scale(dlp, g_loss)
        if dvalues is not None:
            _scale(dvalues, g_loss)
        return (dlp, dvalues) + (None,) * 10


def clip_ratio_loss(
    new_lp: torch.Tensor,
    old_lp: torch.Tensor,
    ref_lp: torch.Tensor | None,
    adv: torch.Tensor,
    response_mask: torch.Tensor,
    rewards: torch.Tensor,
    group_size: int,
    params: N.LossParams,
    ntok: torch.Tensor | None = None,
    whiten: torch.Tensor | None = None,
    values: torch.Tensor | None = None,
    old_values: torch.Tensor | None = None,
):
    """Returns (loss tensor, sums tensor, ntok).  ntok defaults to this call's mask count."""
    dev = N.require_cuda(new_lp, old_lp, ref_lp, adv, response_mask, rewards, values, old_values)
    if new_lp.dim() != 2:
        raise ValueError(f"new_log_probs must be [B, T], got {tuple(new_lp.shape)}")
    B, T = new_lp.shape
    for name, t in (("old_log_probs", old_lp), ("ref_log_probs", ref_lp), ("advantages", adv),
                    ("response_mask", response_mask), ("values", values), ("old_values", old_values)):
        if t is not None and tuple(t.shape) != (B, T):
            raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {(B, T)}")
    m = N.as_mask(response_mask)
    if ntok is None:
        ntok = mask_count(m)
    lp = new_lp if new_lp.dtype in (torch.float32, torch.bfloat16) else new_lp.float()
    loss, sums = ClipRatioLoss.apply(
        lp.contiguous(), None if values is None else values.contiguous().float(),
        old_lp.contiguous().float(), None if ref_lp is None else ref_lp.contiguous().float(),
        adv.contiguous().float(), m, rewards.contiguous().float(), int(group_size), ntok, whiten,
        None if old_values is None else old_values.contiguous().float(), params,
    )
    return loss, sums, ntok


# ---------------------------------------------------------------------------------------------
# SimPO (simpo.py:48-90)
# ---------------------------------------------------------------------------------------------


class SimPOLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, lp, mask_u8, rewards, beta, gamma, chosen_first):
        dev = lp.device
        B, T = lp.shape
        loss = torch.empty((), dtype=torch.float32, device=dev)
        metrics = torch.empty(N.SIMPO_NMETRICS, dtype=torch.float32, device=dev)
        coef = torch.empty(B, dtype=torch.float32, device=dev)
        ws = N.workspace(dev, int(N.lib().ikrl_simpo_workspace_bytes(B)))
        call("ikrl_simpo_fwd", ptr(lp), i32(N.dtype_code(lp)), ptr(mask_u8), ptr(rewards), i32(B), i32(T),
             f32(beta), f32(gamma), i32(1 if chosen_first else 0), ptr(loss), ptr(metrics), ptr(coef), ptr(ws),
             sz(ws.numel()), N.stream_of(dev))
        ctx.save_for_backward(coef, mask_u8)
        ctx.lp_dtype = lp.dtype
        ctx.shape = (B, T)
        ctx.mark_non_differentiable(metrics)
        return loss, metrics

    @staticmethod
    def backward(ctx, g_loss, g_metrics):
        if g_loss is None:
            return (None,) * 6
        coef, m = ctx.saved_tensors
        B, T = ctx.shape
        dlp = torch.empty(B, T, dtype=ctx.lp_dtype, device=coef.device)
        s = g_loss.detach().reshape(1).float().contiguous()
        call("ikrl_simpo_bwd", ptr(coef), ptr(m), i32(B), i32(T), ptr(s), ptr(dlp),
             i32(N.dtype_code(dlp)), N.stream_of(coef.device))
        return dlp, None, None, None, None, None


def simpo_loss(lp, response_mask, rewards, beta, gamma, chosen_first):
    N.require_cuda(lp, response_mask, rewards)
    B, T = lp.shape
    if B % 2:
        raise ValueError(f"SimPO needs an even batch of chosen/rejected pairs, got B={B}")
    x = lp if lp.dtype in (torch.float32, torch.bfloat16) else lp.float()
    return SimPOLoss.apply(x.contiguous(), N.as_mask(response_mask),
                           None if rewards is None else rewards.contiguous().float(), float(beta), float(gamma),
                           bool(chosen_first))


# ---------------------------------------------------------------------------------------------
# K2: logits -> log-prob (policy.py:100-104, :151-155, :187-191)
# ---------------------------------------------------------------------------------------------


class LogitsLogProb(torch.autograd.Function):
    """log p(target) from materialised bf16 logits [N, V] (row stride may exceed V)."""

    @staticmethod
    def forward(ctx, logits, ids):
        dev = logits.device
        Nr, V = logits.shape
        ld = logits.stride(0)
        logp = torch.empty(Nr, dtype=torch.float32, device=dev)
        lse = torch.empty(Nr, dtype=torch.float32, device=dev)
        call("ikrl_logits_logprob_fwd", ptr(logits), i64(ld), ptr(ids), i64(Nr), i32(V), ptr(logp), ptr(lse), None,
             N.stream_of(dev))
        ctx.save_for_backward(logits, ids, lse)
        return logp

    @staticmethod
    def backward(ctx, g):
        logits, ids, lse = ctx.saved_tensors
        Nr, V = logits.shape
        g = g.contiguous().float()
        dlogits = torch.empty(Nr, V, dtype=torch.bfloat16, device=logits.device)
        call("ikrl_logits_logprob_bwd", ptr(logits), i64(logits.stride(0)), ptr(ids), ptr(lse), ptr(g), i64(Nr),
             i32(V), ptr(dlogits), i64(dlogits.stride(0)), N.stream_of(logits.device))
        return dlogits, None


def logits_logprob(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """-F.cross_entropy(logits, targets, reduction="none") over the last dim, as fp32."""
    N.require_cuda(logits, targets)
    if logits.dtype != torch.bfloat16:
        raise TypeError(f"logits_logprob expects bf16 logits, got {logits.dtype}")
    shape = targets.shape
    V = logits.shape[-1]
    x = logits.reshape(-1, V)
    if x.stride(1) != 1:
        x = x.contiguous()
    ids = targets.reshape(-1).to(torch.int64).contiguous()
    return LogitsLogProb.apply(x, ids).reshape(shape)


def logits_logprob_raw(logits: torch.Tensor, ids: torch.Tensor, with_target: bool = False):
    """Forward only: (logp, lse[, gathered target logit]) — used by tests for the bit-exact gather."""
    dev = N.require_cuda(logits, ids)
    Nr, V = logits.shape
    logp = torch.empty(Nr, dtype=torch.float32, device=dev)
    lse = torch.empty(Nr, dtype=torch.float32, device=dev)
    tgt = torch.empty(Nr, dtype=torch.float32, device=dev) if with_target else None
    call("ikrl_logits_logprob_fwd", ptr(logits), i64(logits.stride(0)), ptr(ids), i64(Nr), i32(V), ptr(logp),
         ptr(lse), ptr(tgt), N.stream_of(dev))
    return (logp, lse, tgt) if with_target else (logp, lse)


# ---------------------------------------------------------------------------------------------
# K1: fused LM-head log-prob (policy.py:124-191)
# ---------------------------------------------------------------------------------------------

# bf16 dlogits workspace of one backward chunk (8 GiB: 28,160 rows at V = 151936).  Callers that
# want another size pass chunk_rows; set_ds_chunk_bytes changes the default for the process.
DEFAULT_DS_CHUNK_BYTES = 8 << 30


def set_ds_chunk_bytes(nbytes: int) -> int:
    """Default bytes of the backward's dlogits chunk for later calls; returns the previous value."""
    global DEFAULT_DS_CHUNK_BYTES
    if nbytes < (1 << 20):
        raise ValueError(f"dlogits chunk of {nbytes} bytes is too small")
    prev, DEFAULT_DS_CHUNK_BYTES = DEFAULT_DS_CHUNK_BYTES, int(nbytes)
    return prev


def default_chunk_rows(N: int, V: int, budget_bytes: int | None = None) -> int:
    """Rows per backward chunk so that one chunk of bf16 dlogits fits `budget_bytes`."""
    if budget_bytes is None:
        budget_bytes = DEFAULT_DS_CHUNK_BYTES
    lds = (V + 63) // 64 * 64
    rows = max(128, (budget_bytes // (2 * lds)) // 128 * 128)
    return min(N, rows) if N > rows else N


class LogitCache:
    """Softmax numerators the forward stored for up to `rows` rows (bf16, relative to each
    32-column chunk's maximum) and those maxima (fp32), with each row's slot (-1: not cached).
    The backward forms the cached rows' dlogits from it instead of recomputing their logits."""

    def __init__(self, n_rows: int, V: int, rows: int, device):
        q_el, m_el = N.c_int64(0), N.c_int64(0)
        call("ikrl_lmhead_cache_row_elems", i32(V), N.byref(q_el), N.byref(m_el))
        self.rows = int(rows)
        self.q = torch.empty(self.rows, q_el.value, dtype=torch.bfloat16, device=device)
        self.m = torch.empty(self.rows, m_el.value, dtype=torch.float32, device=device)
        self.slot = torch.empty(n_rows, dtype=torch.int32, device=device)

    @staticmethod
    def bytes_per_row(V: int) -> int:
        q_el, m_el = N.c_int64(0), N.c_int64(0)
        call("ikrl_lmhead_cache_row_elems", i32(V), N.byref(q_el), N.byref(m_el))
        return 2 * q_el.value + 4 * m_el.value


# How much device memory the autograd op may give the logit cache: "auto" uses up to `fraction`
# of the memory free at the forward, after the backward's workspace and outputs and `reserve_bytes`
# are set aside; "off" never caches (the backward recomputes the logits of every active row).
# The cache pays where a row's recompute (2 H V FLOPs) outweighs storing and re-reading its V
# numerators: on B200 the Qwen3-8B head (H = 4096) step ran 17% faster with it, the Qwen3-0.6B
# head (H = 1024) 9% slower, so "auto" caches from H = 2048 (min_hidden).
_LOGIT_CACHE = {"mode": "auto", "reserve_bytes": 4 << 30, "fraction": 0.9, "min_rows": 1024, "min_hidden": 2048}
# Cache rows and candidate rows of the last forward that needed a gradient (for reports).
LOGIT_CACHE_STATS = {"rows": 0, "candidates": 0}


def set_logit_cache(mode: str = "auto", reserve_bytes: int | None = None, fraction: float | None = None) -> dict:
    """Set the logit-cache policy of `lmhead_logprob`; returns the previous one."""
    if mode not in ("auto", "off"):
        raise ValueError(f"logit cache mode {mode!r} is not 'auto' or 'off'")
    prev = dict(_LOGIT_CACHE)
    _LOGIT_CACHE["mode"] = mode
    if reserve_bytes is not None:
        _LOGIT_CACHE["reserve_bytes"] = int(reserve_bytes)
    if fraction is not None:
        _LOGIT_CACHE["fraction"] = float(fraction)
    return prev


def logit_cache_rows(n_rows: int, H: int, V: int, device, candidates: int, chunk_rows: int | None = None) -> int:
    """Cache rows the policy allows for a forward of n_rows rows with `candidates` cacheable rows."""
    if _LOGIT_CACHE["mode"] == "off" or V % 8 or candidates <= 0 or H < _LOGIT_CACHE["min_hidden"]:
        return 0
    free, _ = torch.cuda.mem_get_info(device)
    free += torch.cuda.memory_reserved(device) - torch.cuda.memory_allocated(device)
    if chunk_rows is None:
        chunk_rows = default_chunk_rows(n_rows, V)
    bwd = int(N.lib().ikrl_lmhead_bwd_workspace_bytes(n_rows, H, V, chunk_rows, N.IKRL_DTYPE_BF16, 0))
    outputs = n_rows * H * 2 + V * H * 2  # dhidden and dweight of the backward
    avail = (free - bwd - outputs - _LOGIT_CACHE["reserve_bytes"]) * _LOGIT_CACHE["fraction"]
    rows = min(candidates, max(0, int(avail) // LogitCache.bytes_per_row(V)))
    return rows if rows >= _LOGIT_CACHE["min_rows"] else 0


def lmhead_forward_raw(hidden: torch.Tensor, weight: torch.Tensor, ids: torch.Tensor,
                       cache: LogitCache | None = None, cache_mask: torch.Tensor | None = None):
    """(logp [N] fp32, lse [N] fp32) of the fused kernel; hidden [N, H] and weight [V, H] bf16.
    With `cache`, the forward also fills it for rows where `cache_mask` (bool [N]; all rows when
    None) is set, in row order until its rows are used."""
    dev = N.require_cuda(hidden, weight, ids)
    Nr, H = hidden.shape
    V = weight.shape[0]
    logp = torch.empty(Nr, dtype=torch.float32, device=dev)
    lse = torch.empty(Nr, dtype=torch.float32, device=dev)
    if cache is None:
        nbytes = int(N.lib().ikrl_lmhead_fwd_workspace_bytes(Nr, H, V))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        call("ikrl_lmhead_logprob_fwd", ptr(hidden), ptr(weight), ptr(ids), i64(Nr), i32(H), i32(V), ptr(logp),
             ptr(lse), ptr(ws), sz(nbytes), N.stream_of(dev))
    else:
        m8 = None if cache_mask is None else N.as_mask(cache_mask.reshape(-1))
        nbytes = int(N.lib().ikrl_lmhead_cache_fwd_workspace_bytes(Nr, H, V))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        call("ikrl_lmhead_logprob_fwd_cached", ptr(hidden), ptr(weight), ptr(ids), i64(Nr), i32(H), i32(V),
             ptr(logp), ptr(lse), ptr(m8), i64(cache.rows), ptr(cache.slot), ptr(cache.q), ptr(cache.m), ptr(ws),
             sz(nbytes), N.stream_of(dev))
    if _CHECK_DEVICE_STATUS:
        lmhead_status(ws)
    return logp, lse


def lmhead_backward_raw(hidden, weight, ids, lse, dlogp, want_dh=True, want_dw=True, dw_dtype=torch.bfloat16,
                        chunk_rows: int | None = None, dweight_out: torch.Tensor | None = None,
                        cache: LogitCache | None = None):
    """(dhidden bf16 [N, H] | None, dweight [V, H] | None) for upstream dlogp [N] fp32; `cache` is
    the LogitCache the forward filled, if any."""
    dev = N.require_cuda(hidden, weight, ids, lse, dlogp)
    Nr, H = hidden.shape
    V = weight.shape[0]
    if chunk_rows is None:
        chunk_rows = default_chunk_rows(Nr, V)
    dh = torch.empty_like(hidden) if want_dh else None
    accumulate = 0
    if want_dw:
        if dweight_out is not None:
            dw = dweight_out
            accumulate = 1
        else:
            dw = torch.empty(V, H, dtype=dw_dtype, device=dev)
    else:
        dw = None
    dcode = N.IKRL_DTYPE_F32 if (dw is not None and dw.dtype == torch.float32) else N.IKRL_DTYPE_BF16
    nbytes = int(N.lib().ikrl_lmhead_bwd_workspace_bytes(Nr, H, V, chunk_rows, dcode, accumulate))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    if cache is None:
        call("ikrl_lmhead_logprob_bwd", ptr(hidden), ptr(weight), ptr(ids), ptr(lse), ptr(dlogp), i64(Nr), i32(H),
             i32(V), i64(chunk_rows), ptr(dh), ptr(dw), i32(dcode), i32(accumulate), ptr(ws), sz(nbytes),
             N.stream_of(dev))
    else:
        call("ikrl_lmhead_logprob_bwd_cached", ptr(hidden), ptr(weight), ptr(ids), ptr(lse), ptr(dlogp), i64(Nr),
             i32(H), i32(V), i64(chunk_rows), ptr(dh), ptr(dw), i32(dcode), i32(accumulate), ptr(cache.slot),
             ptr(cache.q), ptr(cache.m), ptr(ws), sz(nbytes), N.stream_of(dev))
    if _CHECK_DEVICE_STATUS:
        lmhead_status(ws)
    return dh, dw


def lmhead_status(ws: torch.Tensor) -> None:
    """Raise if a tensor-core kernel that used `ws` recorded a device-side error (synchronises)."""
    st = N.c_int32(0)
    call("ikrl_lmhead_status", ptr(ws), N.byref(st), N.stream_of(ws.device))


# When set (set_check_device_status), every tensor-core call reads its device status word
# afterwards and raises on a recorded fault; this synchronises the host once per call.
_CHECK_DEVICE_STATUS = False


def set_check_device_status(enable: bool) -> bool:
    global _CHECK_DEVICE_STATUS
    prev, _CHECK_DEVICE_STATUS = _CHECK_DEVICE_STATUS, bool(enable)
    return prev


class LMHeadLogProb(torch.autograd.Function):
    """log p(targets) of hidden @ weight.T without materialising the logits; fp32 output.

    When a gradient is needed and memory allows (`set_logit_cache`), the forward also keeps a
    logit cache for the rows in `cache_rows` (bool [N]; every row when None), so the backward
    forms their dlogits from it instead of recomputing the logits; it is freed by the backward."""

    @staticmethod
    def forward(ctx, hidden, weight, ids, chunk_rows, cache_rows, grad_mode):
        cache = None
        # grad_mode: whether gradients were being recorded at the call (forward itself runs without)
        if grad_mode and (ctx.needs_input_grad[0] or ctx.needs_input_grad[1]):
            Nr, H = hidden.shape
            V = weight.shape[0]
            cand = Nr if cache_rows is None else int(cache_rows.sum())  # one host read per forward
            rows = logit_cache_rows(Nr, H, V, hidden.device, cand, chunk_rows)
            if rows > 0:
                cache = LogitCache(Nr, V, rows, hidden.device)
            LOGIT_CACHE_STATS.update(rows=rows, candidates=cand)
        logp, lse = lmhead_forward_raw(hidden, weight, ids, cache, cache_rows)
        ctx.save_for_backward(hidden, weight, ids, lse)
        ctx.chunk_rows = chunk_rows
        ctx.cache = cache
        return logp

    @staticmethod
    def backward(ctx, g):
        hidden, weight, ids, lse = ctx.saved_tensors
        want_dh, want_dw = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        cache, ctx.cache = ctx.cache, None
        if not (want_dh or want_dw):
            return None, None, None, None, None, None
        dh, dw = lmhead_backward_raw(hidden, weight, ids, lse, g.contiguous().float(), want_dh, want_dw,
                                     weight.dtype if weight.dtype == torch.float32 else torch.bfloat16,
                                     ctx.chunk_rows, cache=cache)
        return dh, dw, None, None, None, None


def lmhead_logprob(hidden: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor,
                   chunk_rows: int | None = None, cache_rows: torch.Tensor | None = None) -> torch.Tensor:
    """Fused F.linear(hidden, weight) + log-softmax gather: hidden [..., H], targets [...] -> fp32 [...].
    Targets of -100 give 0 (ignored rows).  `cache_rows` (bool, shaped like targets) names the rows
    that may carry a gradient, for the logit cache; rows outside it are recomputed in the backward if
    they do (results are the same either way)."""
    N.require_cuda(hidden, weight, targets)
    H = hidden.shape[-1]
    shape = targets.shape
    h = hidden.reshape(-1, H)
    if h.dtype != torch.bfloat16:
        h = h.to(torch.bfloat16)
    if not h.is_contiguous():
        h = h.contiguous()
    w = weight if weight.dtype == torch.bfloat16 else weight.to(torch.bfloat16)
    if not w.is_contiguous():
        w = w.contiguous()
    ids = targets.reshape(-1).to(torch.int64).contiguous()
    if h.shape[0] != ids.shape[0]:
        raise ValueError(f"{h.shape[0]} hidden rows but {ids.shape[0]} targets")
    cr = None
    if cache_rows is not None:
        cr = cache_rows.reshape(-1)
        if cr.shape[0] != ids.shape[0]:
            raise ValueError(f"cache_rows has {cr.shape[0]} entries for {ids.shape[0]} rows")
        cr = cr.to(device=h.device, dtype=torch.bool).contiguous()
    return LMHeadLogProb.apply(h, w, ids, chunk_rows, cr, torch.is_grad_enabled()).reshape(shape)


# ---------------------------------------------------------------------------------------------
# DPO (dpo.py:51-106)
# ---------------------------------------------------------------------------------------------


class DPOLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, lp, ref, mask_u8, rewards, beta, smoothing, chosen_first):
        dev = lp.device
        B, T = lp.shape
        loss = torch.empty((), dtype=torch.float32, device=dev)
        metrics = torch.empty(N.SIMPO_NMETRICS, dtype=torch.float32, device=dev)
        coef = torch.empty(B, dtype=torch.float32, device=dev)
        ws = N.workspace(dev, int(N.lib().ikrl_dpo_workspace_bytes(B)))
        call("ikrl_dpo_fwd", ptr(lp), i32(N.dtype_code(lp)), ptr(ref), ptr(mask_u8), ptr(rewards), i32(B), i32(T),
             f32(beta), f32(smoothing), i32(1 if chosen_first else 0), ptr(loss), ptr(metrics), ptr(coef), ptr(ws),
             sz(ws.numel()), N.stream_of(dev))
        ctx.save_for_backward(coef, mask_u8)
        ctx.lp_dtype = lp.dtype
        ctx.shape = (B, T)
        ctx.mark_non_differentiable(metrics)
        return loss, metrics

    @staticmethod
    def backward(ctx, g_loss, g_metrics):
        if g_loss is None:
            return (None,) * 7
        coef, m = ctx.saved_tensors
        B, T = ctx.shape
        dlp = torch.empty(B, T, dtype=ctx.lp_dtype, device=coef.device)
        s = g_loss.detach().reshape(1).float().contiguous()
        call("ikrl_simpo_bwd", ptr(coef), ptr(m), i32(B), i32(T), ptr(s), ptr(dlp), i32(N.dtype_code(dlp)),
             N.stream_of(coef.device))
        return dlp, None, None, None, None, None, None


def dpo_loss(lp, ref_lp, response_mask, rewards, beta, label_smoothing, chosen_first):
    N.require_cuda(lp, ref_lp, response_mask, rewards)
    B, T = lp.shape
    if B % 2:
        raise ValueError(f"DPO needs an even batch of chosen/rejected pairs, got B={B}")
    x = lp if lp.dtype in (torch.float32, torch.bfloat16) else lp.float()
    return DPOLoss.apply(x.contiguous(), ref_lp.contiguous().float(), N.as_mask(response_mask),
                         None if rewards is None else rewards.contiguous().float(), float(beta),
                         float(label_smoothing), bool(chosen_first))
