"""invokerl_b200 — B200-native (sm_100a) kernels behind invokerl's training hot path.

Drop-in surface (same names and signatures as the reference):
  * ``invokerl_b200.algorithms``: RolloutBatch, BaseAlgorithm, GRPO, DAPO, PPO, SimPO
  * ``invokerl_b200.policy``: PolicyModel.forward / forward_no_grad / _chunked_lm_head_ce /
    _chunk_ce_fn on the fused LM-head kernel
  * ``invokerl_b200.ops``: the autograd functions over the C ABI (include/invokerl_b200.h)
"""

from . import _native, ops  # noqa: F401
from .algorithms import DAPO, DPO, GRPO, PPO, BaseAlgorithm, RolloutBatch, SimPO  # noqa: F401

__version__ = "0.1.0"
