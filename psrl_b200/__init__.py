"""psrl_b200: an asynchronous RL post-training framework for NVIDIA B200.

Layers (bottom-up):

* ``psrl_b200.ops`` / ``psrl_b200.csrc``: hand-written sm_100a kernels and their
  PyTorch reference implementations.
* ``psrl_b200.models``: Qwen2/Qwen2.5/Qwen3 dense and Qwen3-MoE decoders.
* ``psrl_b200.parallel``: process groups, sharded data parallel, tensor and
  expert parallel layers, peer-memory weight sync.
* ``psrl_b200.ps``: the Parameter Server (version binding, staleness inventory).
* ``psrl_b200.rollout``: paged-KV rollout engine, router, coordinator.
* ``psrl_b200.agent`` / ``psrl_b200.reward``: agent loops, data, rewards.
* ``psrl_b200.trainer``: algorithms, actor/critic workers, the RL driver.
"""

__version__ = "0.1.0"
