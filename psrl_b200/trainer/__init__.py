"""Trainer: RL algorithms, actor/critic workers, the RL driver.

``RLTrainer`` and ``compute_batch_advantages`` are loaded on first use, so
that modules the driver itself imports (the agent-loop manager needs
``trainer.batch``) can be imported on their own without a cycle.
"""

__all__ = ["RLTrainer", "compute_batch_advantages"]


def __getattr__(name):
    if name in __all__:
        from . import driver
        return getattr(driver, name)
    raise AttributeError(name)
