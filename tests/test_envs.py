"""Environment registry and the shell-task environment (per-episode
workspace, fenced bash commands, graded by the task's test command), its
reward through the ``env`` reward loop, and workspace cleanup."""

import os

from psrl_b200.agent.data import CharTokenizer
from psrl_b200.agent.envs import ENVIRONMENTS, ShellTaskEnv, make_environment
from psrl_b200.config import load_config
from psrl_b200.reward import RewardManager
from psrl_b200.trainer.batch import Trajectory

TOK = CharTokenizer(1024)
TASK = {"files": {"calc.py": "def add(a, b):\n    return a - b\n"},
        "test_cmd": "python3 -c 'import calc; assert calc.add(2, 3) == 5'"}


def _turn(text):
    return TOK.encode(text)


def test_registry():
    assert {"synthetic_tokens", "tool_env", "shell_env"} <= set(ENVIRONMENTS)
    env = make_environment("shell_env", tokenizer=TOK, max_turns=3)
    assert isinstance(env, ShellTaskEnv)


def test_fix_and_submit_scores_one(tmp_path):
    env = ShellTaskEnv(TOK, max_turns=4, workdir_root=str(tmp_path))
    env.reset(TASK)
    ws = env.ws
    obs, done, info = env.step(0, _turn("I'll fix it.\n```bash\nsed -i 's/a - b/a + b/' calc.py && cat calc.py\n```"))
    text = TOK.decode(obs)
    assert not done and info["returncode"] == 0 and "a + b" in text and "<returncode>0</returncode>" in text
    obs, done, info = env.step(1, _turn("echo COMPLETE_TASK_AND_SUBMIT"))
    assert done and obs == [] and info["reward"] == 1.0 and info["submitted"] == 1.0
    env.close()
    assert not os.path.exists(ws)


def test_unfixed_task_scores_zero_and_commands_time_out(tmp_path):
    env = ShellTaskEnv(TOK, max_turns=2, timeout_s=0.5, workdir_root=str(tmp_path))
    env.reset(TASK)
    obs, done, info = env.step(0, _turn("```bash\nsleep 5\n```"))
    assert not done and info["returncode"] == 124 and "timed out" in TOK.decode(obs)
    obs, done, info = env.step(1, _turn("```bash\nls\n```"))       # out of turns: graded
    assert done and info["reward"] == 0.0
    env.close()


def test_env_reward_loop():
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["reward.kind=env"])
    m = RewardManager(cfg, TOK)
    t = Trajectory(uid=0, request_id=0, prompt_ids=[5], response_ids=[6], rollout_logprobs=[0.0],
                   meta={"env_info": {"reward": 1.0, "commands": 3.0}})
    assert m.score(t) == {"score": 1.0, "commands": 3.0}


def test_multi_turn_loop_closes_workspaces(tmp_path):
    from psrl_b200.agent.loops import MultiTurnAgentLoop
    from psrl_b200.rollout.engine import RequestOutput
    envs = []

    def factory():
        envs.append(ShellTaskEnv(TOK, max_turns=3, workdir_root=str(tmp_path)))
        return envs[-1]

    loop = MultiTurnAgentLoop(factory, lambda rid, turn: 16, max_turns=3)
    o = RequestOutput(request_id=7, prompt_ids=[5, 6], output_ids=_turn("```bash\necho hi\n```"), logprobs=[0.0] * 20,
                      versions=[0] * 20, finish_reason="stop", version_tag=0, meta={"uid": 1, **TASK})
    nxt = loop.on_turn_complete(o)
    assert nxt is not None and "hi" in TOK.decode(nxt.prompt_ids)
    ws = envs[0].ws
    assert os.path.exists(os.path.join(ws, "calc.py"))
    o2 = RequestOutput(request_id=7, prompt_ids=nxt.prompt_ids, output_ids=_turn("COMPLETE_TASK_AND_SUBMIT"),
                       logprobs=[0.0] * 24, versions=[0] * 24, finish_reason="stop", version_tag=0, meta=nxt.meta)
    assert loop.on_turn_complete(o2) is None
    smp = loop.finalize(o2)
    assert smp["env_info"]["reward"] == 0.0 and smp["turns"] == 2
    assert not os.path.exists(ws)


def test_colocated_training_with_shell_env():
    import torch
    torch.set_num_threads(2)
    from psrl_b200.trainer import RLTrainer
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["psrl.agentic_rl.max_turns=2", "psrl.agentic_rl.env=shell_env",
                                                         "reward.kind=env", "rollout.max_response_length=12"])
    t = RLTrainer(cfg)
    out = t.fit(1)
    t.stop_rollout()
    assert out[0]["num_trajectories"] == 32
