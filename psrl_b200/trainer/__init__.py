"""Trainer: RL algorithms, actor/critic workers, the RL driver."""

from .driver import RLTrainer, compute_batch_advantages

__all__ = ["RLTrainer", "compute_batch_advantages"]
