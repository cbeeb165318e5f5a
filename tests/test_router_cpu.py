"""Data-parallel router over fake backend apps (CPU): balancing, failover, streaming,
aggregated health and labeled metrics."""
import json

import pytest

fastapi = pytest.importorskip("fastapi")
httpx = pytest.importorskip("httpx")
from fastapi.testclient import TestClient  # noqa: E402


def fake_backend(name, fail=False):
    from fastapi import FastAPI
    from fastapi.responses import PlainTextResponse, StreamingResponse
    app = FastAPI()
    app.state.calls = 0

    @app.post("/v1/completions")
    async def comp(body: dict):
        app.state.calls += 1
        if fail:
            return PlainTextResponse("boom", status_code=500)
        toks = [t + 1 for t in body["prompt"]]
        if body.get("stream"):
            async def gen():
                for t in toks:
                    yield "data: " + json.dumps({"choices": [{"token_ids": [t]}], "backend": name}) + "\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        return {"choices": [{"token_ids": toks}], "backend": name}

    @app.post("/v1/chat/completions")
    async def chat(body: dict):
        app.state.calls += 1
        return {"object": "chat.completion", "choices": [{"message": {"role": "assistant",
                                                                      "content": body["messages"][-1]["content"][::-1]}}],
                "backend": name}

    @app.get("/health")
    def health():
        return {"status": "ok", "running": 0}

    @app.get("/metrics")
    def metrics():
        return PlainTextResponse("# TYPE steps_total counter\nsteps_total 7\nlat_bucket{le=\"1\"} 3\n")
    return app


def _router(apps, **kw):
    from rocket_b200.serve_router import Backend, build_router
    bs = [Backend(f"b{i}", httpx.AsyncClient(transport=httpx.ASGITransport(app=a), base_url=f"http://b{i}"))
          for i, a in enumerate(apps)]
    return bs, TestClient(build_router(bs, **kw))


def test_balances_and_fails_over():
    a0, a1 = fake_backend("b0"), fake_backend("b1")
    bs, c = _router([a0, a1])
    for i in range(6):
        r = c.post("/v1/completions", json={"prompt": [i, i + 1]})
        assert r.status_code == 200 and r.json()["choices"][0]["token_ids"] == [i + 1, i + 2]
    assert a0.state.calls == 3 and a1.state.calls == 3      # alternates under light load
    bad, good = fake_backend("bad", fail=True), fake_backend("good")
    bs, c = _router([bad, good], cooldown_s=60)
    r = c.post("/v1/completions", json={"prompt": [1]})
    assert r.status_code == 200 and r.json()["backend"] == "good"
    assert bs[0].failed == 1 and not bs[0].up()
    c.post("/v1/completions", json={"prompt": [1]})
    assert bad.state.calls == 1                              # marked down: not tried again


def test_stream_health_metrics_and_auth():
    bs, c = _router([fake_backend("b0"), fake_backend("b1")], api_key="k")
    assert c.post("/v1/completions", json={"prompt": [1]}).status_code == 401
    hdr = {"Authorization": "Bearer k"}
    with c.stream("POST", "/v1/completions", json={"prompt": [4, 5], "stream": True}, headers=hdr) as s:
        ev = [ln[6:] for ln in s.iter_lines() if ln.startswith("data: ")]
    assert ev[-1] == "[DONE]" and [json.loads(e)["choices"][0]["token_ids"][0] for e in ev[:-1]] == [5, 6]
    assert all(b.inflight == 0 for b in bs)
    h = c.get("/health").json()
    assert h["status"] == "ok" and len(h["backends"]) == 2
    m = c.get("/metrics").text
    assert 'steps_total{backend="b0"} 7' in m and 'lat_bucket{backend="b1",le="1"} 3' in m


def test_chat_is_routed():
    a0, a1 = fake_backend("b0"), fake_backend("b1")
    bs, c = _router([a0, a1])
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "abc"}]})
    assert r.status_code == 200 and r.json()["choices"][0]["message"]["content"] == "cba"
    assert a0.state.calls + a1.state.calls == 1
