"""Rollout packing (invokerl/generator.py:414-455) on the GPU against the reference's own output
and the oracle: bit-exact token ids, log-probs and masks."""

import pytest
import torch

import oracle
from helpers import load
from invokerl_b200.rollout import pack_output

pytestmark = pytest.mark.gpu

FIELDS = ("token_ids", "log_probs", "prompt_mask", "response_mask", "attention_mask")


def test_pack_matches_reference_golden():
    g = load("rollout_pack")
    out = pack_output(g["all_ids"], g["all_lps"], g["prompt_lens"], g["completion_lens"], g["texts"], g["pad_id"])
    for k in FIELDS:
        got = getattr(out, k).cpu()
        assert got.dtype == g[k].dtype, k
        assert torch.equal(got, g[k]), k
    assert out.prompt_lens == g["prompt_lens"] and out.texts == g["texts"]


@pytest.mark.parametrize("B,maxlen", [(1, 1), (3, 300), (64, 2048), (257, 700)])
def test_pack_matches_oracle_random(B, maxlen):
    gen = torch.Generator().manual_seed(B + maxlen)
    ids, lps, pls, cls = [], [], [], []
    for i in range(B):
        p = int(torch.randint(0, maxlen + 1, (1,), generator=gen))
        c = int(torch.randint(0, maxlen - p + 1, (1,), generator=gen))
        ids.append(torch.randint(0, 151936, (p + c,), generator=gen).tolist())
        lp = [0.0] * p + torch.randn(c, generator=gen).tolist()
        lps.append(lp[: len(lp) - (i % 3)] if i % 5 == 0 else lp)
        pls.append(p)
        cls.append(c)
    out = pack_output(ids, lps, pls, cls, [""] * B, pad_id=7)
    want = oracle.pack_rollouts(ids, lps, pls, cls, 7)
    for k in FIELDS:
        assert torch.equal(getattr(out, k).cpu(), want[k]), k


def test_pack_empty_batch():
    out = pack_output([], [], [], [], [], pad_id=0)
    assert out.token_ids.shape == (0, 0) and out.attention_mask.dtype == torch.bool
