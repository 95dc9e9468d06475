"""Vocab-parallel LM-head log-probs: W split along the vocabulary over the ranks of a process
group, hidden rows replicated.

Each rank runs the fused K1 forward on its vocabulary slice and keeps, per row, the slice's
logsumexp and (when the target id is in the slice) the raw target logit.  One all-gather of
these two [N] fp32 vectors gives every rank the global logsumexp and log-probs.  The backward
needs no further exchange for dW (each rank's slice of dW is local); the rank terms of dH are
summed with one all-reduce.  The result equals `ops.lmhead_logprob` on the whole W up to fp32
summation order.  The reference keeps the whole W on every rank; this is the optional
tensor-parallel layout of the same computation.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _native as N
from .ops import default_chunk_rows, lmhead_status
from . import ops as _ops


def _world(group):
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def shard_forward_raw(hidden, weight_shard, ids, vocab_start: int):
    """(tlogit [N], lse_shard [N]) fp32 of this rank's vocabulary slice."""
    dev = N.require_cuda(hidden, weight_shard, ids)
    Nr, H = hidden.shape
    Vs = weight_shard.shape[0]
    tl = torch.empty(Nr, dtype=torch.float32, device=dev)
    ls = torch.empty(Nr, dtype=torch.float32, device=dev)
    nbytes = int(N.lib().ikrl_lmhead_fwd_workspace_bytes(Nr, H, Vs))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    N.call("ikrl_lmhead_shard_fwd", N.ptr(hidden), N.ptr(weight_shard), N.ptr(ids), N.i64(Nr), N.i32(H), N.i32(Vs),
           N.i64(vocab_start), N.ptr(tl), N.ptr(ls), N.ptr(ws), N.sz(nbytes), N.stream_of(dev))
    if _ops._CHECK_DEVICE_STATUS:
        lmhead_status(ws)
    return tl, ls


def combine(parts: torch.Tensor, ids: torch.Tensor, vocab_size: int):
    """(logp [N], lse [N]) from the ranks' [P, 2, N] (tlogit, lse_shard)."""
    P, two, Nr = parts.shape
    assert two == 2
    logp = torch.empty(Nr, dtype=torch.float32, device=parts.device)
    lse = torch.empty(Nr, dtype=torch.float32, device=parts.device)
    N.call("ikrl_vocab_parallel_combine", N.ptr(parts.contiguous()), N.ptr(ids), N.i64(Nr), N.i32(P),
           N.i64(vocab_size), N.ptr(logp), N.ptr(lse), N.stream_of(parts.device))
    return logp, lse


def shard_backward_raw(hidden, weight_shard, ids, lse, dlogp, vocab_start: int, want_dh=True, want_dw=True,
                       dw_dtype=torch.bfloat16, chunk_rows: int | None = None):
    """(this rank's dH term bf16 [N, H] | None, this rank's dW slice [V_shard, H] | None)."""
    dev = N.require_cuda(hidden, weight_shard, ids, lse, dlogp)
    Nr, H = hidden.shape
    Vs = weight_shard.shape[0]
    if chunk_rows is None:
        chunk_rows = default_chunk_rows(Nr, Vs)
    dh = torch.empty_like(hidden) if want_dh else None
    dw = torch.empty(Vs, H, dtype=dw_dtype, device=dev) if want_dw else None
    dcode = N.IKRL_DTYPE_F32 if (dw is not None and dw.dtype == torch.float32) else N.IKRL_DTYPE_BF16
    nbytes = int(N.lib().ikrl_lmhead_bwd_workspace_bytes(Nr, H, Vs, chunk_rows, dcode, 0))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    N.call("ikrl_lmhead_shard_bwd", N.ptr(hidden), N.ptr(weight_shard), N.ptr(ids), N.ptr(lse), N.ptr(dlogp),
           N.i64(Nr), N.i32(H), N.i32(Vs), N.i64(vocab_start), N.i64(chunk_rows), N.ptr(dh), N.ptr(dw),
           N.i32(dcode), N.i32(0), N.ptr(ws), N.sz(nbytes), N.stream_of(dev))
    if _ops._CHECK_DEVICE_STATUS:
        lmhead_status(ws)
    return dh, dw


class VocabParallelLMHeadLogProb(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight_shard, ids, vocab_start, vocab_size, group, chunk_rows):
        P, _ = _world(group)
        tl, ls = shard_forward_raw(hidden, weight_shard, ids, vocab_start)
        local = torch.stack([tl, ls])
        if P > 1:
            parts = torch.empty(P, 2, local.shape[1], dtype=torch.float32, device=local.device)
            dist.all_gather_into_tensor(parts, local, group=group)
        else:
            parts = local.unsqueeze(0)
        logp, lse = combine(parts, ids, vocab_size)
        ctx.save_for_backward(hidden, weight_shard, ids, lse)
        ctx.vocab_start, ctx.group, ctx.chunk_rows, ctx.P = vocab_start, group, chunk_rows, P
        return logp

    @staticmethod
    def backward(ctx, g):
        hidden, weight_shard, ids, lse = ctx.saved_tensors
        want_dh, want_dw = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        # every rank takes part in the dH all-reduce, so each computes its term
        dh, dw = shard_backward_raw(hidden, weight_shard, ids, lse, g.contiguous().float(), ctx.vocab_start,
                                    True, want_dw,
                                    weight_shard.dtype if weight_shard.dtype == torch.float32 else torch.bfloat16,
                                    ctx.chunk_rows)
        if ctx.P > 1:
            acc = dh.float()
            dist.all_reduce(acc, group=ctx.group)
            dh = acc.to(hidden.dtype)
        return (dh if want_dh else None), dw, None, None, None, None, None


def lmhead_logprob_vocab_parallel(hidden: torch.Tensor, weight_shard: torch.Tensor, targets: torch.Tensor,
                                  vocab_start: int, vocab_size: int, group=None,
                                  chunk_rows: int | None = None) -> torch.Tensor:
    """log p(targets) of hidden @ W.T (fp32, shape of targets) with W split over `group` along the
    vocabulary: this rank holds rows [vocab_start, vocab_start + weight_shard.shape[0]) of the
    vocab_size rows.  Every rank passes the same hidden rows and targets and gets the same
    log-probs; the gradient of weight_shard is this rank's slice of dW."""
    N.require_cuda(hidden, weight_shard, targets)
    H = hidden.shape[-1]
    shape = targets.shape
    h = hidden.reshape(-1, H)
    h = h if h.dtype == torch.bfloat16 else h.to(torch.bfloat16)
    h = h if h.is_contiguous() else h.contiguous()
    w = weight_shard if weight_shard.dtype == torch.bfloat16 else weight_shard.to(torch.bfloat16)
    w = w if w.is_contiguous() else w.contiguous()
    ids = targets.reshape(-1).to(torch.int64).contiguous()
    return VocabParallelLMHeadLogProb.apply(h, w, ids, int(vocab_start), int(vocab_size), group,
                                            chunk_rows).reshape(shape)


def shard_bounds(vocab_size: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's vocabulary slice.  The vocabulary is cut into blocks of 8 rows
    (16-byte aligned W rows); the blocks are dealt out contiguously and as evenly as possible, so
    slice sizes differ by at most 15 rows (8 from the uneven deal, 7 from a vocabulary that is not
    a multiple of 8).  A slice is empty only when vocab_size < 8 * world."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    blocks = -(-vocab_size // 8)
    base, extra = divmod(blocks, world)
    start = 8 * (rank * base + min(rank, extra))
    end = 8 * ((rank + 1) * base + min(rank + 1, extra))
    return min(vocab_size, start), min(vocab_size, end)
