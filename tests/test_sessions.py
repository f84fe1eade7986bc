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
