"""Reward plane: reward functions, reward-loop registry, normalisation, the
generative reward model (C19)."""

from .functions import REWARD_LOOPS, RewardManager, addition_score, bernoulli_hash_score, register_reward_loop
from .loops import (GEN_RM_FUNCTIONS, EngineRewardModel, HttpRewardModel, default_compute_score,
                    gen_reward_function, last_boxed)

__all__ = ["REWARD_LOOPS", "RewardManager", "addition_score", "bernoulli_hash_score", "register_reward_loop",
           "GEN_RM_FUNCTIONS", "EngineRewardModel", "HttpRewardModel", "default_compute_score",
           "gen_reward_function", "last_boxed"]
