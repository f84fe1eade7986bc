"""Reward loops: answer scoring, PRIME process-pool scoring with timeouts,
GDPO components into the estimator, and the generative reward model over
the HTTP and rollout-engine services."""

import time

import torch

from psrl_b200.agent.data import CharTokenizer
from psrl_b200.config import load_config
from psrl_b200.reward import EngineRewardModel, HttpRewardModel, RewardManager, default_compute_score, last_boxed
from psrl_b200.trainer import algos
from psrl_b200.trainer.batch import Trajectory
from psrl_b200.trainer.driver import compute_batch_advantages
from psrl_b200.utils.common import HttpPostPool

TOK = CharTokenizer(1024)


def slow_score(data_source, solution_str, ground_truth, extra_info=None):
    time.sleep(3.0)
    return 1.0


def two_part_score(data_source, solution_str, ground_truth, extra_info=None):
    return {"acc": float(str(ground_truth) in solution_str), "format": 0.5 if "####" in solution_str else 0.0}


def _traj(text, answer, rid=0, uid=0, prompt="What is 40 + 2?"):
    return Trajectory(uid=uid, request_id=rid, prompt_ids=TOK.encode(prompt), response_ids=TOK.encode(text),
                      rollout_logprobs=[0.0] * len(TOK.encode(text)), meta={"answer": answer})


def _mgr(kind, *ov, reward_model=None):
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[f"reward.kind={kind}", *ov])
    return RewardManager(cfg, TOK, reward_model=reward_model)


def test_boxed_and_default_scores():
    assert last_boxed("so \\boxed{\\frac{1}{2}} and \\boxed{7}") == "7"
    assert last_boxed("x = \\boxed{\\frac{1}{2}}") == "\\frac{1}{2}"
    assert last_boxed("no box") is None
    assert default_compute_score("addition", "it is #### 42", 42) == 1.0
    assert default_compute_score("addition", "it is #### 41", 42) == 0.0
    assert default_compute_score("math", "thus \\boxed{1,000}", "1000") == 1.0
    assert default_compute_score("math", "thus \\boxed{x+1}", "x + 1") == 1.0
    assert default_compute_score("other", "Paris", "Paris") == 1.0


def test_prime_scores_in_processes_and_times_out():
    m = _mgr("prime", "reward.num_processes=2")
    assert m.score(_traj("#### 42", 42))["score"] == 1.0
    assert m.score(_traj("#### 7", 42))["score"] == 0.0
    m.close()
    slow = _mgr("prime", "reward.num_processes=1", "reward.timeout_s=0.5",
                "reward.compute_score=tests.test_reward_loops:slow_score")
    r = slow.score(_traj("#### 42", 42))
    assert r["score"] == 0.0 and r["timeout"] == 1.0
    scorer = slow.ctx["_prime"]
    first_pool = scorer.pool
    r = slow.score(_traj("#### 42", 42))            # the stuck worker was replaced
    assert r["timeout"] == 1.0 and scorer.stats["timeouts"] == 2 and scorer.pool is not first_pool
    slow.close()


def test_gdpo_components_reach_the_estimator():
    m = _mgr("gdpo", "reward.compute_score=tests.test_reward_loops:two_part_score")
    trajs = []
    for i, (txt, uid) in enumerate([("#### 42", 0), ("42", 0), ("nope", 0), ("#### 42", 1), ("#### 1", 1)]):
        t = _traj(txt, 42, rid=i, uid=uid)
        sc = m.score(t)
        t.reward = sc["score"]
        t.meta["reward_extra"] = sc
        trajs.append(t)
    assert trajs[0].meta["reward_extra"]["components"] == [1.0, 0.5]
    assert trajs[0].reward == 1.5
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["algorithm.adv_estimator=gdpo"])
    compute_batch_advantages(cfg, trajs)
    comps = torch.tensor([t.meta["reward_extra"]["components"] for t in trajs])
    want = algos.gdpo_advantage(comps, [t.uid for t in trajs])
    torch.testing.assert_close(torch.tensor([t.advantage for t in trajs]), want)


class _FakeRM:
    def __init__(self, verdict):
        self.verdict = verdict
        self.prompts = []

    def generate(self, prompt_ids):
        self.prompts.append(TOK.decode(prompt_ids))
        return f"The steps check out. \\boxed{{{self.verdict}}}"


def test_gen_reward_model_judges_with_template():
    rm = _FakeRM("True")
    m = _mgr("gen", reward_model=rm)
    assert m.score(_traj("#### 42", 42))["score"] == 1.0
    p = rm.prompts[0]
    assert "What is 40 + 2?" in p and "#### 42" in p and p.startswith("<|im_start|>user")
    assert _mgr("gen", reward_model=_FakeRM("False")).score(_traj("#### 42", 42))["score"] == 0.0
    sc = _mgr("gen", "reward.gen_rm.function=scalar", reward_model=_FakeRM("7")).score(_traj("x", 1))
    assert abs(sc["score"] - 0.7) < 1e-9


def test_gen_reward_model_over_http():
    seen = []

    def post(url, payload, timeout):
        seen.append((url, payload))
        return {"choices": [{"text": "\\boxed{True}"}]}

    rm = HttpRewardModel("http://rm.local:8000/", TOK, max_tokens=64, pool=HttpPostPool(post=post))
    m = _mgr("gen", reward_model=rm)
    assert m.score(_traj("#### 42", 42))["score"] == 1.0
    assert seen[0][0] == "http://rm.local:8000/v1/completions" and seen[0][1]["max_tokens"] == 64


def test_gen_reward_model_on_engine_replicas():
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.rollout import EngineWeights, RolloutEngine
    a = PRESETS["tiny"]
    engines = []
    for s in range(2):
        mdl = build_model(a, "cpu", torch.float32, seed=s)
        engines.append(RolloutEngine(a, EngineWeights.from_model(mdl, "cpu", torch.float32), max_num_seqs=4,
                                     max_model_len=1024, block_size=16, kv_cache_gb=0.05, use_cuda_graph=False))
    rm = EngineRewardModel(engines, TOK, max_tokens=8)
    m = _mgr("gen", reward_model=rm)
    for i in range(3):
        assert m.score(_traj("#### 42", 42, rid=i))["score"] in (0.0, 1.0)
    assert all(not e.has_unfinished() for e in engines)


def test_gen_reward_model_built_from_config():
    m = _mgr("gen", "reward.gen_rm.preset=tiny", "reward.gen_rm.replicas=2", "reward.gen_rm.max_tokens=4",
             "reward.gen_rm.kv_cache_gb=0.05", "++reward.gen_rm.max_model_len=1024", "trainer.device=cpu")
    rm = m.ctx["reward_model"]
    assert isinstance(rm, EngineRewardModel) and len(rm.engines) == 2
    assert m.score(_traj("#### 42", 42))["score"] in (0.0, 1.0)
