"""Reward plane: reward functions, reward-loop registry, normalisation (C19)."""

from .functions import REWARD_LOOPS, RewardManager, addition_score, bernoulli_hash_score, register_reward_loop

__all__ = ["REWARD_LOOPS", "RewardManager", "addition_score", "bernoulli_hash_score", "register_reward_loop"]
