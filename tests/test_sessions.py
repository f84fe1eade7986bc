from psrl_b200.rollout.session_router import SessionRouter
from psrl_b200.rollout.session_scheduler import SessionInfo, ThunderAgentScheduler


def _gen(prompt, n, tag, inst):
    return [7] * n, [-0.5] * n, [3] * n, (tag if tag >= 0 else 3), inst or (1, 0)


def test_session_router_http_roundtrip():
    from fastapi.testclient import TestClient
    r = SessionRouter(_gen)
    c = TestClient(r.app())
    a = c.post("/v1/sessions/s1/completions", json={"prompt_ids": [1, 2], "max_tokens": 2}).json()
    assert a["output_ids"] == [7, 7] and a["version_tag"] == 3
    b = c.post("/v1/sessions/s1/completions", json={"prompt_ids": [1, 2, 7, 7, 9], "max_tokens": 1}).json()
    assert b["version_tag"] == 3
    assert c.post("/control/hang", json={"session_ids": ["s1"]}).json() == {"hung": ["s1"]}
    assert c.post("/v1/sessions/s1/completions", json={"prompt_ids": [1], "max_tokens": 1}).status_code == 409
    c.post("/control/continue", json={"session_ids": ["s1"]})
    assert c.get("/sessions").json()["s1"]["turns"] == 2
    smp = c.post("/v1/sessions/s1/close").json()
    assert smp["response_ids"] == [7, 7, 9, 7] and smp["response_mask"] == [1, 1, 0, 1]


def test_thunder_agent_hang_and_continue():
    sch = ThunderAgentScheduler(capacity_tokens=1000, env_token_weight=1.0, buffer_per_session=0)
    ss = [SessionInfo("a", 400, "gen"), SessionInfo("b", 300, "env", 100), SessionInfo("c", 350, "gen")]
    hang, cont = sch.decide(ss)
    assert hang == ["b"] and cont == []                # env sessions are hung first
    ss = [SessionInfo("a", 400, "gen"), SessionInfo("b", 500, "hung"), SessionInfo("c", 200, "hung"),
          SessionInfo("d", 300, "hung")]
    hang, cont = sch.decide(ss)
    assert hang == [] and cont == ["b"]               # best fit decreasing: 500 fits 600 free


def test_session_agent_loop_on_engines():
    import torch

    from psrl_b200.agent.loops import SessionAgentLoop
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.rollout import EngineWeights, RolloutEngine
    from psrl_b200.rollout.session_router import engine_generate_fn
    a = PRESETS["tiny"]
    engines = []
    for v in (4, 5):
        m = build_model(a, "cpu", torch.float32, seed=v)
        e = RolloutEngine(a, EngineWeights.from_model(m, "cpu", torch.float32), max_num_seqs=4, max_model_len=512,
                          block_size=16, kv_cache_gb=0.05, use_cuda_graph=False)
        e.version = v
        engines.append(e)
    router = SessionRouter(engine_generate_fn(engines))

    def agent(client, task):
        ctx = list(task["prompt"])
        for turn in range(3):
            out = client.complete(ctx, 4)
            ctx = ctx + out + [9, 9]          # tool observation between turns
        if task.get("fail"):
            raise ValueError("agent crashed")

    loop = SessionAgentLoop(router, agent, workers=3)
    res = loop.run([{"prompt": [5, 6, 7]}, {"prompt": [8, 8]}, {"prompt": [3], "fail": True}])
    assert len(res) == 3 and not router.sessions
    for r in res:
        assert len(r["response_ids"]) == 3 * 4 + 2 * 2
        assert r["response_mask"] == [1] * 4 + [0, 0] + [1] * 4 + [0, 0] + [1] * 4
        assert r["version_tag"] in (4, 5)           # pinned to the first turn's engine version
    assert res[2]["error"].startswith("ValueError")

    trajs = SessionAgentLoop.to_trajectories(res, uid=3, request_id_base=30)
    assert len(trajs) == 2 and [t.request_id for t in trajs] == [30, 31]
    assert all(t.uid == 3 and t.response_len == 16 and len(t.rollout_logprobs) == 16 for t in trajs)


def test_session_router_runs_the_capacity_scheduler():
    """With a ThunderAgent scheduler in the router, a session over capacity is
    hung at a turn boundary (its next turn answers 409), and closing another
    session continues it; a local client waits through the hang."""
    import threading
    sch = ThunderAgentScheduler(capacity_tokens=50, env_token_weight=1.0, buffer_per_session=0)
    r = SessionRouter(_gen, scheduler=sch)
    r.complete("a", [1] * 20, 5)                       # a: 25 tokens, in env
    r.complete("b", [1] * 20, 5)                       # b: 25 tokens -> 50 used, fits
    out = r.complete("c", [1] * 10, 5)                 # c pushes the total over 50: an env session is hung
    assert "output_ids" in out and r.sched_stats["hung"] >= 1
    hung = [k for k, v in r.states().items() if v["hung"]]
    assert hung
    assert r.complete(hung[0], [1] * 30, 1).get("status") == 409
    from psrl_b200.rollout.session_router import LocalSessionClient
    got = {}
    t = threading.Thread(target=lambda: got.update(ids=LocalSessionClient(r, hung[0]).complete([1] * 30, 1)))
    t.start()
    for k in [k for k in ("a", "b", "c") if k != hung[0]]:
        r.close(k)                                     # frees capacity: the hung session continues
    t.join(timeout=10)
    assert got.get("ids") == [7] and r.sched_stats["continued"] >= 1
