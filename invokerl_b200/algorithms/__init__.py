"""Drop-in algorithm classes with invokerl's interface (invokerl/algorithms/__init__.py)."""

from .base import BaseAlgorithm, RolloutBatch
from .dapo import DAPO
from .dpo import DPO
from .grpo import GRPO
from .ppo import PPO
from .simpo import SimPO

__all__ = ["BaseAlgorithm", "RolloutBatch", "GRPO", "DPO", "PPO", "SimPO", "DAPO"]
