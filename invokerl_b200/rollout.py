"""Rollout packing on the GPU: the padded tensors of a generation call.

`pack_output` has the arguments and result of invokerl's `VLLMGenerator._pack_output`
(invokerl/generator.py:414-455): per-sequence token ids (prompt + completion) and per-token
log-probs (0 for prompt tokens) become [B, T] tensors plus prompt / response / attention masks,
T = the longest sequence.  The reference builds each row with host `torch.tensor(...)` calls;
here the ragged lists are concatenated once, copied to the device in one transfer per field, and
one kernel (`ikrl_pack_rollouts`) writes every row.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from . import _native as N


@dataclass
class GenerationOutput:
    """Output of a generation call (invokerl/generator.py:39-49, same fields)."""

    token_ids: Tensor  # [B, T] int64, prompt + completion, padded with pad_id
    prompt_lens: list[int]
    completion_lens: list[int]
    log_probs: Tensor  # [B, T] fp32, 0 for prompt tokens and padding
    texts: list[str]
    prompt_mask: Tensor  # [B, T] bool
    response_mask: Tensor  # [B, T] bool
    attention_mask: Tensor  # [B, T] bool


def _csr(rows, dtype) -> tuple[Tensor, Tensor]:
    lens = torch.tensor([len(r) for r in rows], dtype=torch.int64)
    offsets = torch.zeros(len(rows) + 1, dtype=torch.int64)
    torch.cumsum(lens, 0, out=offsets[1:])
    flat = [x for r in rows for x in r]
    values = torch.tensor(flat, dtype=dtype) if flat else torch.zeros(1, dtype=dtype)
    return values, offsets


def pack_output(all_ids: list[list[int]], all_lps: list[list[float]], prompt_lens: list[int],
                completion_lens: list[int], texts: list[str], pad_id: int,
                device: str | torch.device = "cuda") -> GenerationOutput:
    """Pad variable-length outputs into fixed-size tensors on `device` (generator.py:414-455)."""
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError("invokerl_b200.rollout.pack_output runs on a CUDA device; there is no CPU path")
    B = len(all_ids)
    T = max((len(ids) for ids in all_ids), default=0)
    ids_v, ids_o = _csr(all_ids, torch.int64)
    lps_v, lps_o = _csr(all_lps, torch.float32)
    host = [ids_v, ids_o, lps_v, lps_o, torch.tensor(prompt_lens, dtype=torch.int32).reshape(B),
            torch.tensor(completion_lens, dtype=torch.int32).reshape(B)]
    d = [t.pin_memory().to(dev, non_blocking=True) for t in host]
    token_ids = torch.empty(B, T, dtype=torch.int64, device=dev)
    log_probs = torch.empty(B, T, dtype=torch.float32, device=dev)
    masks = [torch.empty(B, T, dtype=torch.bool, device=dev) for _ in range(3)]
    if B and T:
        N.call("ikrl_pack_rollouts", *(N.ptr(t) for t in d), N.i32(B), N.i32(T), N.i64(pad_id),
               N.ptr(token_ids), N.ptr(log_probs), *(N.ptr(m) for m in masks), N.stream_of(dev))
    return GenerationOutput(token_ids=token_ids, prompt_lens=list(prompt_lens),
                            completion_lens=list(completion_lens), log_probs=log_probs, texts=list(texts),
                            prompt_mask=masks[0], response_mask=masks[1], attention_mask=masks[2])
