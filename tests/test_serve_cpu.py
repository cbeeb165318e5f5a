"""HTTP front-end over a fake engine (CPU): completions, streaming, health, metrics, auth,
greedy-only refusal and engine-fault propagation."""
import json
import time

import pytest

from rocket_b200.engine.scheduler import Request

fastapi = pytest.importorskip("fastapi")
from fastapi.testclient import TestClient  # noqa: E402


class _Sched:
    def __init__(self):
        self.running, self.waiting = [], []

    def has_work(self):
        return bool(self.running or self.waiting)


class FakeEngine:
    """Greedy 'model': the next token is (last + 1) % 1000; one token per step per request."""

    def __init__(self, fail_after=None):
        self.sched = _Sched()
        self.phase = "idle"
        self.steps = 0
        self.fail_after = fail_after

    def add_request(self, prompt, max_new, stop=()):
        r = Request(list(prompt), max_new, tuple(stop))
        self.sched.waiting.append(r)
        return r

    def step(self):
        self.steps += 1
        if self.fail_after is not None and self.steps > self.fail_after:
            self.phase = "faulted"
            raise RuntimeError("injected device failure")
        self.sched.running += self.sched.waiting
        self.sched.waiting = []
        now = time.perf_counter()
        for r in list(self.sched.running):
            nxt = ((r.output[-1] if r.output else r.prompt[-1]) + 1) % 1000
            r.output.append(nxt)
            r.t_tokens.append(now)
            r.t_first = r.t_first or now
            if r.finished():
                r.t_done = now
                self.sched.running.remove(r)


def _client(engine, **kw):
    from rocket_b200.serve import EngineLoop, build_app
    loop = EngineLoop(engine).start()
    return loop, TestClient(build_app(loop, "fake", **kw))


def test_completion_and_stream():
    loop, c = _client(FakeEngine())
    try:
        r = c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 4})
        assert r.status_code == 200, r.text
        body = r.json()
        assert body["choices"][0]["token_ids"] == [8, 9, 10, 11]
        assert body["usage"] == {"prompt_tokens": 3, "completion_tokens": 4, "total_tokens": 7}
        assert body["choices"][0]["finish_reason"] == "length"
        r = c.post("/v1/completions", json={"prompt": [1], "max_tokens": 5, "stop_token_ids": [4]})
        assert r.json()["choices"][0]["token_ids"] == [2, 3, 4] and r.json()["choices"][0]["finish_reason"] == "stop"
        with c.stream("POST", "/v1/completions", json={"prompt": [10], "max_tokens": 3, "stream": True}) as s:
            events = [ln[6:] for ln in s.iter_lines() if ln.startswith("data: ")]
        assert events[-1] == "[DONE]"
        toks = [t for e in events[:-1] for t in json.loads(e)["choices"][0]["token_ids"]]
        assert toks == [11, 12, 13]
        h = c.get("/health").json()
        assert h["status"] == "ok" and h["running"] == 0
        assert c.get("/v1/models").json()["data"][0]["id"] == "fake"
    finally:
        loop.stop()


def test_auth_and_refusals():
    loop, c = _client(FakeEngine(), api_key="secret")
    try:
        assert c.post("/v1/completions", json={"prompt": [1], "max_tokens": 2}).status_code == 401
        hdr = {"Authorization": "Bearer secret"}
        assert c.post("/v1/completions", json={"prompt": [1], "max_tokens": 2}, headers=hdr).status_code == 200
        r = c.post("/v1/completions", json={"prompt": [1], "max_tokens": 2, "temperature": 0.7}, headers=hdr)
        assert r.status_code == 400
        assert c.post("/v1/completions", json={"prompt": "text", "max_tokens": 2}, headers=hdr).status_code == 400
        assert c.post("/v1/completions", json={"prompt": [1], "max_tokens": 0}, headers=hdr).status_code == 400
    finally:
        loop.stop()


def test_engine_fault_reaches_clients():
    loop, c = _client(FakeEngine(fail_after=2))
    try:
        r = c.post("/v1/completions", json={"prompt": [1], "max_tokens": 10})
        assert r.status_code == 503 and "injected" in r.json()["error"]
        assert c.get("/health").json()["status"] == "error"
        r = c.post("/v1/completions", json={"prompt": [1], "max_tokens": 3})
        assert r.status_code == 503
    finally:
        loop.stop()


def _follow_worker(rank, port, q):
    import asyncio
    import datetime

    import torch.distributed as dist

    from rocket_b200.serve import EngineLoop, follow
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=60))
    eng = FakeEngine()
    try:
        if rank == 0:
            class Par:
                world = 2
            loop = EngineLoop(eng, Par()).start()

            async def go():
                ps = [loop.submit([i * 10], 3, (), asyncio.get_running_loop()) for i in range(3)]
                outs = []
                for p in ps:
                    got = []
                    while True:
                        item = await p.queue.get()
                        if item is None:
                                break
                        got += item
                    outs.append(got)
                return outs
            outs = asyncio.run(go())
            loop.stop()
            q.put((0, outs, eng.steps))
        else:
            follow(eng)
            q.put((1, [r.output for r in eng.sched.running], eng.steps))
    finally:
        dist.destroy_process_group()


def test_rank0_serves_followers_step_in_lockstep():
    import socket

    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_follow_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict((r, (o, st)) for r, o, st in (q.get(timeout=120) for _ in range(2)))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][0] == [[1, 2, 3], [11, 12, 13], [21, 22, 23]]
    assert res[0][1] == res[1][1]  # the same number of engine steps on both ranks


class ByteTok:
    """Token i -> byte i (a byte-level vocabulary): multi-byte UTF-8 characters span tokens."""

    def encode(self, text):
        return list(text.encode("utf-8"))

    def decode(self, ids):
        return bytes(i % 256 for i in ids).decode("utf-8", errors="replace")


class EchoEngine(FakeEngine):
    """Emits the bytes of a fixed UTF-8 string, one per step."""

    def __init__(self, text):
        super().__init__()
        self.payload = list(text.encode("utf-8"))

    def step(self):
        self.sched.running += self.sched.waiting
        self.sched.waiting = []
        now = time.perf_counter()
        for r in list(self.sched.running):
            r.output.append(self.payload[len(r.output) % len(self.payload)])
            r.t_first = r.t_first or now
            if r.finished():
                r.t_done = now
                self.sched.running.remove(r)


def test_streamed_text_never_splits_a_character():
    from rocket_b200.serve import EngineLoop, build_app
    text = "ok é 漢字 ✓"
    n = len(text.encode("utf-8"))
    loop = EngineLoop(EchoEngine(text)).start()
    try:
        c = TestClient(build_app(loop, "fake", tokenizer=ByteTok()))
        with c.stream("POST", "/v1/completions", json={"prompt": "x", "max_tokens": n, "stream": True}) as s:
            ev = [json.loads(ln[6:]) for ln in s.iter_lines() if ln.startswith("data: ") and ln != "data: [DONE]"]
        parts = [e["choices"][0]["text"] for e in ev]
        assert "".join(parts) == text
        assert all("�" not in p for p in parts)
        r = c.post("/v1/completions", json={"prompt": "x", "max_tokens": n})
        assert r.json()["choices"][0]["text"] == text
    finally:
        loop.stop()


def test_chat_completions():
    """Messages go through the chat template; the reply ends at the eos token, which the
    text leaves out; streaming opens with the role and sends content deltas."""
    from rocket_b200.serve import EngineLoop, build_app, render_chat
    seen = []

    class RecordingEcho(EchoEngine):
        def add_request(self, prompt, max_new, stop=()):
            seen.append((list(prompt), tuple(stop)))
            return super().add_request(prompt, max_new, stop)

    loop = EngineLoop(RecordingEcho("hi é!")).start()
    try:
        tpl = "{% for m in messages %}[{{ m['role'] }}]{{ m['content'] }}{% endfor %}[assistant]"
        c = TestClient(build_app(loop, "fake", tokenizer=ByteTok(), chat_template=tpl, eos_ids=[ord("!")]))
        msgs = [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hello"}]
        r = c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 20})
        assert r.status_code == 200, r.text
        body = r.json()
        assert body["object"] == "chat.completion"
        ch = body["choices"][0]
        assert ch["message"] == {"role": "assistant", "content": "hi é"} and ch["finish_reason"] == "stop"
        assert bytes(seen[-1][0]).decode() == "[system]be brief[user]hello[assistant]"
        assert ord("!") in seen[-1][1]
        with c.stream("POST", "/v1/chat/completions", json={"messages": msgs, "max_tokens": 20, "stream": True}) as s:
            ev = [json.loads(ln[6:]) for ln in s.iter_lines() if ln.startswith("data: ") and ln != "data: [DONE]"]
        assert ev[0]["choices"][0]["delta"] == {"role": "assistant"}
        assert all(e["object"] == "chat.completion.chunk" for e in ev)
        assert "".join(e["choices"][0]["delta"].get("content", "") for e in ev[1:]) == "hi é"
        assert ev[-1]["choices"][0]["finish_reason"] == "stop"
        assert c.post("/v1/chat/completions", json={"messages": "nope"}).status_code == 400
        assert "<|user|>\nhello\n<|assistant|>\n" in render_chat([{"role": "user", "content": "hello"}])
    finally:
        loop.stop()
    loop2 = EngineLoop(FakeEngine()).start()
    try:
        c2 = TestClient(build_app(loop2, "fake"))
        assert c2.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}]}).status_code == 400
    finally:
        loop2.stop()


class AbortableEngine(FakeEngine):
    """FakeEngine with abort(), slowed so a request is still running when it is cancelled."""

    def __init__(self):
        super().__init__()
        self.aborted = []

    def step(self):
        time.sleep(0.01)
        super().step()

    def abort(self, req):
        self.aborted.append(req)
        if req in self.sched.running:
            self.sched.running.remove(req)
        if req in self.sched.waiting:
            self.sched.waiting.remove(req)


def test_cancel_aborts_the_request_and_ends_its_stream():
    import asyncio

    from rocket_b200.serve import EngineLoop
    eng = AbortableEngine()
    loop = EngineLoop(eng).start()

    async def go():
        p = loop.submit([1], 10_000, (), asyncio.get_running_loop())
        got = []
        while len(got) < 3:
            got += await asyncio.wait_for(p.queue.get(), 10)
        loop.cancel(p)
        while True:
            item = await asyncio.wait_for(p.queue.get(), 10)
            if item is None:
                return p, got
    try:
        p, got = asyncio.run(go())
        assert eng.aborted == [p.req] and loop.aborted == 1 and len(p.req.output) < 10_000
        assert not eng.sched.has_work()
    finally:
        loop.stop()


def test_full_queue_answers_429():
    import threading

    from rocket_b200.serve import EngineLoop, QueueFull, build_app
    gate = threading.Event()

    class Blocked(FakeEngine):
        def step(self):
            gate.wait(10)
            super().step()

    eng = Blocked()
    loop = EngineLoop(eng, max_pending=3).start()  # the admitted request still counts as waiting
    try:
        c = TestClient(build_app(loop, "fake"))
        import asyncio
        ev = asyncio.new_event_loop()
        ps = [loop.submit([1], 2, (), ev)]      # admitted: the loop thread blocks in step()
        time.sleep(0.2)
        ps += [loop.submit([2], 2, (), ev), loop.submit([3], 2, (), ev)]
        with pytest.raises(QueueFull):
            loop.submit([4], 2, (), ev)
        r = c.post("/v1/completions", json={"prompt": [5], "max_tokens": 2})
        assert r.status_code == 429 and r.headers.get("retry-after") == "1"
    finally:
        gate.set()
        loop.stop()


def _cancel_worker(rank, port, q):
    import asyncio
    import datetime

    import torch.distributed as dist

    from rocket_b200.serve import EngineLoop, follow
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=60))
    eng = AbortableEngine()
    try:
        if rank == 0:
            class Par:
                world = 2
            loop = EngineLoop(eng, Par()).start()

            async def go():
                keep = loop.submit([100], 30, (), asyncio.get_running_loop())
                drop = loop.submit([500], 10_000, (), asyncio.get_running_loop())
                got = []
                while len(got) < 3:
                    got += await asyncio.wait_for(drop.queue.get(), 20)
                loop.cancel(drop)
                out = []
                while True:
                    item = await asyncio.wait_for(keep.queue.get(), 20)
                    if item is None:
                        return out
                    out += item
            out = asyncio.run(go())
            loop.stop()
            q.put((0, [r.prompt for r in eng.aborted], eng.steps, len(out)))
        else:
            follow(eng)
            q.put((1, [r.prompt for r in eng.aborted], eng.steps, None))
    finally:
        dist.destroy_process_group()


def test_cancellation_reaches_every_rank():
    import socket

    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_cancel_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {r: (ab, st, n) for r, ab, st, n in (q.get(timeout=120) for _ in range(2))}
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][0] == res[1][0] == [[500]]   # the same request aborted on both ranks
    assert res[0][1] == res[1][1] and res[0][2] == 30
