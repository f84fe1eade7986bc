"""Multi-turn agent loops, environments, tool parsers and the TITO builder."""

import pytest

from psrl_b200.agent.envs import SyntheticTokenEnv, ToolEnv
from psrl_b200.agent.tito import TurnRecord, build_training_data
from psrl_b200.agent.tool_parser import get_parser
from psrl_b200.agent.tools import FunctionTool, ToolRegistry


def test_tool_parsers():
    c, rest = get_parser("hermes")('hi <tool_call>{"name": "add", "arguments": {"a": 1}}</tool_call>')
    assert c[0].name == "add" and c[0].arguments == {"a": 1} and rest == "hi"
    c, _ = get_parser("xml_fc")("<function_call><name>f</name><arguments>{\"x\": 2}</arguments></function_call>")
    assert c[0].name == "f" and c[0].arguments == {"x": 2}
    c, _ = get_parser("qwen3_coder")("<tool_call><function=run><parameter=n>3</parameter>"
                                     "<parameter=s>abc</parameter></function></tool_call>")
    assert c[0].name == "run" and c[0].arguments == {"n": 3, "s": "abc"}
    c, _ = get_parser("gpt_oss")("<|start|>assistant<|channel|>commentary to=functions.lookup <|message|>"
                                 "{\"q\": \"x\"}<|call|>")
    assert c[0].name == "lookup" and c[0].arguments == {"q": "x"}
    c, _ = get_parser("gemma4")("```tool_code\nsearch(q='cats', k=2)\n```")
    assert c[0].name == "search" and c[0].arguments == {"q": "cats", "k": 2}
    with pytest.raises(KeyError):
        get_parser("nope")


def test_tool_env_runs_tools():
    from psrl_b200.agent.data import CharTokenizer
    tok = CharTokenizer(1024)
    reg = ToolRegistry([FunctionTool(lambda a, b: int(a) + int(b), name="add")])
    env = ToolEnv(tok, reg, "hermes", max_turns=3)
    obs, done, info = env.step(0, tok.encode('<tool_call>{"name": "add", "arguments": {"a": 2, "b": 5}}</tool_call>'))
    assert not done and "7" in tok.decode(obs) and info["num_calls"] == 1
    obs, done, _ = env.step(1, tok.encode("the answer is 7"))
    assert done and obs == []


def test_tito_builder_masks_env_tokens():
    t0 = TurnRecord([1, 2, 3], [10, 11], [-0.1, -0.2], [0, 0])
    t1 = TurnRecord([1, 2, 3, 10, 11, 50, 51, 52], [12], [-0.3], [1])
    smp = build_training_data([t0, t1])
    assert smp.prompt_ids == [1, 2, 3]
    assert smp.response_ids == [10, 11, 50, 51, 52, 12]
    assert smp.response_mask == [1, 1, 0, 0, 0, 1]
    assert smp.rollout_logprobs == [-0.1, -0.2, 0.0, 0.0, 0.0, -0.3]
    assert smp.turn_count == 2
    with pytest.raises(ValueError):
        build_training_data([t0, TurnRecord([9, 9], [1], [0.0])])


def test_synthetic_env_is_deterministic():
    e = SyntheticTokenEnv(1000, max_turns=3, obs_lo=5, obs_hi=9, seed=1)
    e.reset({"uid": 2, "request_id": 9})
    a, d0, _ = e.step(0, [1])
    e.reset({"uid": 2, "request_id": 9})
    b, _, _ = e.step(0, [1])
    assert a == b and 5 <= len(a) <= 9 and not d0
    assert e.step(2, [1])[1]


def test_multiturn_rl_cpu():
    from psrl_b200.config import load_config
    from psrl_b200.trainer import RLTrainer
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[
        "psrl.agentic_rl.max_turns=3", "++psrl.agentic_rl.obs_len_min=4", "++psrl.agentic_rl.obs_len_max=8",
        "data.kind=synthetic_tokens", "data.prompt_len_min=8", "data.prompt_len_max=16",
        "data.response_len_mu=1.5", "data.response_len_sigma=0.3", "data.response_len_cap=8",
        "reward.kind=bernoulli_hash", "rollout.ignore_eos=true", "rollout.block_size=4",
        "psrl.staleness_buffer_entries=4", "actor.ppo_mini_batch_size=4"])
    t = RLTrainer(cfg)
    m = t.step()
    assert m["num_trajectories"] == 16
    assert t.engine.bm.hits > 0                      # later turns reuse the session prefix
    t2 = t.step()
    assert t2["num_trajectories"] == 16


@pytest.mark.parametrize("scope", ["recompute", "pre_step"])
def test_fine_grain_overlap_strategy_cpu(scope):
    from psrl_b200.config import load_config
    from psrl_b200.trainer import RLTrainer
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[
        "psrl.fine_grain_overlap.granularity=mini_batch", f"psrl.fine_grain_overlap.overlap_scope={scope}",
        "actor.ppo_mini_batch_size=4", "psrl.log_prob.enable_rollout_engine_log_prob=false",
        "rollout.max_response_length=8"])
    t = RLTrainer(cfg)
    m = t.step()
    assert m["num_trajectories"] == 32 and m["fine_grain/chunks"] == 2
    assert all(tr is not None for tr in [m.get("actor/pg_loss")])
