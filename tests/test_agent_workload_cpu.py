"""Forked-prefix agent traces (generation, causality check, KV-sharing summary), their
replay through a backend, and the HTTP load generator against the real server over a
socket (fake engine, CPU)."""
import json
import socket
import subprocess
import sys
import threading
import time

import pytest

from rocket_b200.engine.agent_workload import (Completion, agent_trace, kv_costs, replay_trace, trace_summary,
                                               validate_trace)


def test_trace_is_valid_seeded_and_shares_prefixes():
    ev = agent_trace(concurrency=8, depth=2, prefix_tokens=2048, duration_steps=300, seed=3)
    assert validate_trace(ev) == []
    assert ev == agent_trace(concurrency=8, depth=2, prefix_tokens=2048, duration_steps=300, seed=3)
    assert ev != agent_trace(concurrency=8, depth=2, prefix_tokens=2048, duration_steps=300, seed=4)
    kinds = {e["event"] for e in ev}
    assert {"session_start", "prefill", "decode", "idle", "resume", "session_end"} <= kinds
    assert {e["kind"] for e in ev if e["event"] == "prefill"} == {"root", "fork", "tool"}
    depths = {e["depth"] for e in ev if e["event"] == "session_start"}
    assert depths == {0, 1, 2}
    per_tick = {}
    for e in ev:
        if e["event"] == "decode":
            per_tick[e["t"]] = per_tick.get(e["t"], 0) + 1
    assert max(per_tick.values()) <= 8
    s = trace_summary(ev, kv_bytes_per_token=100, fixed_bytes_per_session=7)
    assert s["total_tokens"] == s["inherited_tokens"] + s["fresh_tokens"]
    assert 0.5 < s["prefix_shared_fraction"] < 1.0
    assert s["kv_bytes_with_sharing"] < s["kv_bytes_without_sharing"]
    assert s["kv_bytes_without_sharing"] == 100 * s["total_tokens"] + 7 * s["sessions"]
    assert s["peak_concurrent_decoding"] == 8


def test_trace_respects_max_context():
    ev = agent_trace(concurrency=4, depth=2, prefix_tokens=500, duration_steps=400, seed=1, max_context=900)
    assert validate_trace(ev) == []
    ctx = {}
    for e in ev:
        if e["event"] == "session_start":
            ctx[e["session"]] = e["fork_point_tokens"]
        elif e["event"] in ("prefill", "decode"):
            ctx[e["session"]] += e["n_tokens"]
            if e["session"] != "s0":
                assert ctx[e["session"]] <= 900


def test_validate_flags_causality_errors():
    ev = agent_trace(concurrency=2, depth=1, prefix_tokens=64, duration_steps=30, seed=0)
    bad = [dict(e) for e in ev]
    first_decode = next(i for i, e in enumerate(bad) if e["event"] == "decode")
    sid = bad[first_decode]["session"]
    start = next(i for i, e in enumerate(bad) if e["event"] == "session_start" and e["session"] == sid)
    bad[start]["session"] = "ghost"
    assert any("not live" in m for m in validate_trace(bad))
    bad = [dict(e) for e in ev]
    bad[3]["seq"] = 0
    assert any("backwards" in m for m in validate_trace(bad))
    bad = [dict(e) for e in ev] + [{"t": 10 ** 6, "seq": 10 ** 6, "event": "resume", "session": "s1"}]
    assert validate_trace(bad)


class _EchoBackend:
    """Completion = the next `n` integers after the prompt's last token; records prompts."""

    def __init__(self):
        self.prompts = []

    def run_batch(self, jobs):
        out = []
        for p, n in jobs:
            self.prompts.append(list(p))
            now = time.perf_counter()
            out.append(Completion([(p[-1] + 1 + i) % 1000 for i in range(n)], now, now, [now] * n, cached=len(p) // 2))
        return out


def test_replay_builds_histories_from_forks():
    ev = agent_trace(concurrency=4, depth=2, prefix_tokens=128, duration_steps=60, seed=2)
    be = _EchoBackend()
    res = replay_trace(be, ev, vocab=1000, seed=0)
    n_dec = sum(1 for e in ev if e["event"] == "decode")
    assert res["requests"] == n_dec == len(be.prompts)
    assert res["output_tokens"] == sum(e["n_tokens"] for e in ev if e["event"] == "decode")
    # every session's prompt starts with the root prefix (the fork chain copies it)
    root_prefix = be.prompts[0][:128]
    assert all(p[:128] == root_prefix for p in be.prompts)
    # prompt length = the trace's context before each decode
    ctx, lens = {}, []
    for e in ev:
        if e["event"] == "session_start":
            ctx[e["session"]] = e["fork_point_tokens"]
        elif e["event"] == "prefill":
            ctx[e["session"]] += e["n_tokens"]
        elif e["event"] == "decode":
            lens.append(ctx[e["session"]])
            ctx[e["session"]] += e["n_tokens"]
    assert sorted(lens) == sorted(len(p) for p in be.prompts)
    assert res["prompt_cache_fraction"] == pytest.approx(
        sum(len(p) // 2 for p in be.prompts) / sum(len(p) for p in be.prompts), abs=1e-4)


def test_kv_costs_of_the_fuels():
    from rocket_b200.config import load_fuel
    cfg = load_fuel("glm-moe-355b").model
    per_tok, fixed = kv_costs(cfg)
    n_attn = cfg.num_layers
    assert per_tok == n_attn * 2 * cfg.num_kv_heads * cfg.head_dim * 2 and fixed == 0
    assert kv_costs(cfg, "fp8")[0] == per_tok // 2
    hy = load_fuel("qwen3-next-hybrid").model
    per_tok, fixed = kv_costs(hy)
    assert fixed > 0 and per_tok > 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.fixture
def live_server():
    pytest.importorskip("fastapi")
    uvicorn = pytest.importorskip("uvicorn")
    sys.path.insert(0, __file__.rsplit("/", 1)[0])
    from test_serve_cpu import FakeEngine

    from rocket_b200.serve import EngineLoop, build_app
    loop = EngineLoop(FakeEngine()).start()
    port = _free_port()
    server = uvicorn.Server(uvicorn.Config(build_app(loop, "fake"), host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    t0 = time.time()
    while not server.started and time.time() - t0 < 30:
        time.sleep(0.05)
    assert server.started
    yield f"http://127.0.0.1:{port}"
    server.should_exit = True
    th.join(timeout=10)
    loop.stop()


def test_http_client_streams_and_replays(live_server):
    from rocket_b200.engine.loadgen import poisson_workload
    from rocket_b200.serve_client import HttpBackend, run_http_open_loop, stream_completion
    c = stream_completion(live_server, [5, 6], 4)
    assert c.tokens == [7, 8, 9, 10] and c.t_first is not None and len(c.t_tokens) == 4
    wl = poisson_workload(12, 200.0, (3, 9), 4, 1000, seed=1, max_out=6)
    res = run_http_open_loop(live_server, wl, max_inflight=4)
    assert res["completed"] == 12 and res["errors"] == 0
    assert res["output_tokens"] == sum(a.max_new_tokens for a in wl)
    ev = agent_trace(concurrency=3, depth=1, prefix_tokens=32, duration_steps=8, seed=0)
    be = HttpBackend(live_server, max_inflight=4)
    try:
        r = replay_trace(be, ev, vocab=1000)
    finally:
        be.close()
    assert r["output_tokens"] == sum(e["n_tokens"] for e in ev if e["event"] == "decode")


def test_agent_trace_cli(tmp_path):
    out = tmp_path / "t.jsonl"
    cmd = [sys.executable, "-m", "rocket_b200", "agent-trace", "--fuel", "glm-moe-small", "--concurrency", "4",
           "--duration-steps", "50", "--prefix-tokens", "256", "--out", str(out)]
    subprocess.run(cmd, check=True, timeout=300)
    lines = [json.loads(x) for x in out.read_text().splitlines()]
    assert lines[-1]["event"] == "summary" and lines[-1]["kv_bytes_per_token"] > 0
    r = subprocess.run([sys.executable, "-m", "rocket_b200", "agent-trace", "--validate", "--trace", str(out)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and json.loads(r.stdout)["valid"]


def test_agent_trace_cli_rejects_a_broken_trace(tmp_path):
    ev = agent_trace(concurrency=2, depth=1, prefix_tokens=32, duration_steps=20, seed=1)
    ev = [e for e in ev if not (e["event"] == "session_start" and e["session"] == "s1")]  # orphan events
    p = tmp_path / "bad.jsonl"
    p.write_text("\n".join(json.dumps(e) for e in ev) + "\n")
    r = subprocess.run([sys.executable, "-m", "rocket_b200", "agent-trace", "--validate", "--trace", str(p)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 1 and not json.loads(r.stdout)["valid"] and "not live" in r.stderr
