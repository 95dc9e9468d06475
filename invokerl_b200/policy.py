"""PolicyModel with invokerl's interface (invokerl/policy.py:17-196) and the fused LM-head kernel.

`forward` keeps the reference's contract — per-token log-probs [B, T] with position 0 equal to
zero and position t holding log p(token_ids[t] | token_ids[<t]) — but the LM head + log-softmax +
gather run as one tcgen05 kernel that never materialises the [B*T, V] logits (the reference
loops over 64-token chunks under torch.utils.checkpoint).  Log-probs are returned in float32
(the reference returns the hidden dtype, bf16 by default).  Under FSDP the wrapped model still
produces full logits (policy.py:90-105); those go through the one-pass logits kernel instead of
F.cross_entropy.  Model loading, FSDP wrapping and vLLM weight sharing stay with the reference.
"""

from __future__ import annotations

import contextlib

import torch
from torch import Tensor

from . import ops


class PolicyModel:
    """Wraps a HuggingFace CausalLM; forward() returns per-token log-probs with gradients."""

    def __init__(
        self,
        model_name_or_path: str,
        device: str = "cuda",
        dtype: torch.dtype = torch.bfloat16,
        master_weights_fp32: bool = False,
    ):
        from transformers import AutoModelForCausalLM

        load_dtype = torch.float32 if master_weights_fp32 else dtype
        model = AutoModelForCausalLM.from_pretrained(model_name_or_path, dtype=load_dtype,
                                                     attn_implementation="sdpa").to(device)
        model.train()
        model.config.use_cache = False
        model.gradient_checkpointing_enable()
        self._setup(model, device, dtype, dtype if master_weights_fp32 else None)

    @classmethod
    def from_model(cls, model, device: str | torch.device = "cuda", dtype: torch.dtype = torch.bfloat16,
                   autocast_dtype: torch.dtype | None = None, fsdp_wrapped: bool = False) -> PolicyModel:
        """Wrap an already constructed CausalLM (no download)."""
        self = cls.__new__(cls)
        self._setup(model, device, dtype, autocast_dtype)
        self._fsdp_wrapped = fsdp_wrapped
        return self

    def _setup(self, model, device, dtype, autocast_dtype):
        self.model = model
        self.device = device
        self.dtype = dtype
        self.master_weights_fp32 = autocast_dtype is not None
        self._autocast_dtype = autocast_dtype
        self._fsdp_wrapped = False

    def forward(self, token_ids: Tensor, attention_mask: Tensor, ce_chunk_size: int = 64) -> Tensor:
        """Per-token log-probs [B, T] (fp32); position 0 is 0.  `ce_chunk_size` is accepted for
        interface compatibility; the fused kernel has no logits chunk to size."""
        token_ids = token_ids.to(self.device)
        attention_mask = attention_mask.to(self.device)
        ctx = (torch.autocast("cuda", dtype=self._autocast_dtype) if self._autocast_dtype
               else contextlib.nullcontext())
        with ctx:
            if self._fsdp_wrapped:
                logits = self.model(input_ids=token_ids, attention_mask=attention_mask).logits
                if logits.dtype != torch.bfloat16:
                    logits = logits.to(torch.bfloat16)
                # All T positions as rows of the [B*T, V] logits (a view, no copy of the slice
                # logits[:, :-1]); the last position has no target (-100, log-prob -0.0, no gradient).
                targets = torch.full_like(token_ids, -100)
                targets[:, :-1] = token_ids[:, 1:]
                log_probs = ops.logits_logprob(logits, targets)[:, :-1]
                pad = torch.zeros(token_ids.shape[0], 1, device=log_probs.device, dtype=log_probs.dtype)
                return torch.cat([pad, log_probs], dim=1)
            hidden = self.model.model(input_ids=token_ids, attention_mask=attention_mask).last_hidden_state
        # Every position t < T-1 predicts token t+1; the last position has no target (-100).
        targets = torch.full_like(token_ids, -100)
        targets[:, :-1] = token_ids[:, 1:]
        # Rows whose target is an attended token are the ones a loss can weight (the response
        # tokens among them); they are the candidates for the logit cache of the backward.
        cache_rows = torch.zeros_like(token_ids, dtype=torch.bool)
        cache_rows[:, :-1] = attention_mask[:, 1:].bool()
        lp = ops.lmhead_logprob(hidden, self.model.lm_head.weight, targets, cache_rows=cache_rows)
        pad = torch.zeros(token_ids.shape[0], 1, device=lp.device, dtype=lp.dtype)
        return torch.cat([pad, lp[:, :-1]], dim=1)

    def _chunked_lm_head_ce(self, hidden_states: Tensor, targets: Tensor, chunk_size: int) -> Tensor:
        """LM head + log-prob of `targets` for hidden_states [B, T, H] (policy.py:124-171); fp32."""
        return ops.lmhead_logprob(hidden_states, self.model.lm_head.weight, targets)

    @staticmethod
    def _chunk_ce_fn(lm_head_weight: Tensor, hidden_chunk: Tensor, target_chunk: Tensor) -> Tensor:
        """F.linear + -cross_entropy of one chunk (policy.py:173-191); fp32."""
        return ops.lmhead_logprob(hidden_chunk, lm_head_weight, target_chunk)

    @torch.no_grad()
    def forward_no_grad(self, token_ids: Tensor, attention_mask: Tensor) -> Tensor:
        """forward() without gradients (reference log-probs, policy.py:193-196)."""
        return self.forward(token_ids, attention_mask)
