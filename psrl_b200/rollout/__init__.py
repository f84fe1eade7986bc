"""Rollout plane: paged-KV engine, router, coordinator, sessions."""

from .engine import EngineWeights, GenRequest, RequestOutput, RolloutEngine, SamplingParams

__all__ = ["EngineWeights", "GenRequest", "RequestOutput", "RolloutEngine", "SamplingParams"]
