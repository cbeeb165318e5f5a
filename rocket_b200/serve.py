"""HTTP serving front-end: an OpenAI-style completions API over one engine (or one engine
group spanning several GPUs).

    python -m rocket_b200 serve --fuel glm-moe-355b --port 8000                # 1 GPU
    torchrun --nproc-per-node 8 -m rocket_b200 serve --fuel glm-moe-355b      # TP/EP 8: rank 0 serves

Endpoints:
    POST /v1/completions   {"prompt": str | [ids], "max_tokens": n, "stop_token_ids": [...],
                            "stream": bool}  -> text (with a tokenizer) and token ids; streaming
                            sends one server-sent event per step that produced tokens
    POST /v1/chat/completions  {"messages": [{role, content}], ...}: the messages rendered
                            through the chat template (tokenizer_config.json's, or a
                            default), replies end at the eos token
    GET  /v1/models        the loaded fuel
    GET  /health           engine state (idle / active / faulted), queue depths
    GET  /metrics          Prometheus text (engine counters and latency histograms)

One background thread owns the engine: it admits queued requests, runs `engine.step()`
while there is work, and hands each step's new tokens to the waiting HTTP handlers
(asyncio futures / queues resolved thread-safely).  With several ranks, rank 0 runs the
HTTP server and broadcasts every step's new requests (token ids) before the step, so all
ranks admit the same requests in the same order and step in lockstep; the other ranks
run `follow()` (no HTTP).  A streaming client that disconnects cancels its request (it
leaves the engine on every rank at the next step boundary); with `max_pending`, requests
beyond that many waiting for admission are answered 429.  Only greedy decoding is served (as in the reference engines,
which reject temperature / top-p); requests asking for sampling are refused.

The reference serves through its own CLIs (rocket-decode, rocket-coding-bench) and
measures vLLM / SGLang through their OpenAI APIs (scripts/baseline/openai-forked-prefix.py);
this module gives the engine that API directly.
"""
from __future__ import annotations

import asyncio
import itertools
import json
import threading
import time
from dataclasses import dataclass, field


@dataclass
class _Pending:
    prompt: list
    max_new: int
    stop: tuple
    loop: asyncio.AbstractEventLoop
    queue: asyncio.Queue             # receives lists of new token ids, then None at the end
    req: object = None
    sent: int = 0
    seq: int = -1                    # admission order (the same on every rank)
    t_submit: float = field(default_factory=time.perf_counter)


class QueueFull(RuntimeError):
    """More requests wait for admission than the server accepts (HTTP 429)."""


class EngineLoop:
    """Runs an engine on a background thread; `submit` is safe from any thread."""

    def __init__(self, engine, par=None, idle_sleep_s: float = 0.002, max_pending: int | None = None):
        self.engine = engine
        self.par = par
        self.idle = idle_sleep_s
        self.max_pending = max_pending   # queued + not yet admitted requests; None = unbounded
        self._lock = threading.Lock()
        self._incoming: list[_Pending] = []
        self._cancel: list[_Pending] = []
        self._live: dict[int, _Pending] = {}
        self._admitted = 0
        self.aborted = 0
        self._stop = False
        self.error: str | None = None
        self._thread = threading.Thread(target=self._run, name="rocket-engine", daemon=True)

    def start(self):
        self._thread.start()
        return self

    def stop(self):
        self._stop = True
        self._thread.join(timeout=30)

    def submit(self, prompt, max_new: int, stop=(), loop=None) -> _Pending:
        loop = loop or asyncio.get_event_loop()
        p = _Pending(list(map(int, prompt)), int(max_new), tuple(stop), loop, asyncio.Queue())
        with self._lock:
            if self.error:
                raise RuntimeError(self.error)
            if self.max_pending is not None and \
                    len(self._incoming) + len(self.engine.sched.waiting) >= self.max_pending:
                self._count("requests_rejected_total")
                raise QueueFull(f"{self.max_pending} requests already wait for admission")
            self._incoming.append(p)
        return p

    def cancel(self, p: _Pending):
        """Drop a request whose client went away: it leaves the engine at the next step
        boundary (on every rank) and its stream ends."""
        with self._lock:
            if p in self._incoming:
                self._incoming.remove(p)
                self._deliver(p, None)
            else:
                self._cancel.append(p)

    def _count(self, name: str):
        m = getattr(self.engine, "metrics", None)
        if m is not None:
            m.inc(name)

    def _deliver(self, p: _Pending, item):
        p.loop.call_soon_threadsafe(p.queue.put_nowait, item)

    def _admit(self, batch: list[_Pending]):
        for p in batch:
            p.req = self.engine.add_request(p.prompt, p.max_new, p.stop)
            p.seq = self._admitted
            self._admitted += 1
            self._live[id(p.req)] = p

    def _abort(self, gone: list[_Pending]):
        for p in gone:
            if p.req is not None and id(p.req) in self._live and p.req.t_done is None:
                self.engine.abort(p.req)
                del self._live[id(p.req)]
                self.aborted += 1
                self._count("requests_cancelled_total")
                self._deliver(p, None)

    def _broadcast(self, new: list):
        """World > 1: rank 0's new requests (and the stop flag) reach every rank before the step."""
        import torch.distributed as dist
        box = [new]
        dist.broadcast_object_list(box, src=0)
        return box[0]

    def _run(self):
        eng = self.engine
        multi = self.par is not None and getattr(self.par, "world", 1) > 1
        while True:
            with self._lock:
                batch, self._incoming = self._incoming, []
                gone, self._cancel = self._cancel, []
            gone = [p for p in gone if p.req is not None and id(p.req) in self._live]
            if multi:
                desc = [(p.prompt, p.max_new, p.stop) for p in batch]
                msg = self._broadcast({"new": desc, "abort": [p.seq for p in gone], "stop": self._stop})
                if msg["stop"]:
                    break
            elif self._stop:
                break
            try:
                self._abort(gone)
                self._admit(batch)
                if eng.sched.has_work():
                    eng.step()
                elif not batch:
                    time.sleep(self.idle)
                    continue
            except Exception as e:  # the engine is faulted: fail every waiting request
                self.error = f"{type(e).__name__}: {e}"
                for p in list(self._live.values()) + self._incoming:
                    self._deliver(p, RuntimeError(self.error))
                self._live.clear()
                break
            for key, p in list(self._live.items()):
                out = p.req.output
                if len(out) > p.sent:
                    self._deliver(p, list(out[p.sent:]))
                    p.sent = len(out)
                if p.req.t_done is not None:
                    self._deliver(p, None)
                    del self._live[key]


def follow(engine):
    """Non-zero ranks of a serving group: admit what rank 0 broadcasts, step in lockstep."""
    import torch.distributed as dist
    admitted: dict[int, object] = {}  # admission order -> request (rank 0 names aborts by it)
    while True:
        box = [None]
        dist.broadcast_object_list(box, src=0)
        msg = box[0]
        if msg["stop"]:
            return
        for seq in msg.get("abort", []):
            r = admitted.get(seq)
            if r is not None and r.t_done is None:
                engine.abort(r)
        for prompt, max_new, stop in msg["new"]:
            admitted[len(admitted)] = engine.add_request(prompt, max_new, stop)
        if engine.sched.has_work():
            engine.step()


_ids = itertools.count()


def build_app(loop: EngineLoop, model_name: str, tokenizer=None, api_key: str | None = None,
              max_tokens_limit: int = 4096, chat_template: str | None = None, eos_ids=()):
    """`chat_template`: a Jinja chat template (a tokenizer_config.json's) for
    /v1/chat/completions, else DEFAULT_CHAT_TEMPLATE; `eos_ids` end a chat reply."""
    from fastapi import FastAPI, Header, HTTPException
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    app = FastAPI(title="rocket_b200")

    def _auth(authorization):
        if api_key and authorization != f"Bearer {api_key}":
            raise HTTPException(status_code=401, detail="bad or missing API key")

    def _prompt_ids(body):
        pr = body.get("prompt")
        if isinstance(pr, list) and all(isinstance(x, int) for x in pr):
            return pr
        if isinstance(pr, str):
            if tokenizer is None:
                raise HTTPException(status_code=400, detail="text prompts need a tokenizer (--tokenizer)")
            return tokenizer.encode(pr)
        raise HTTPException(status_code=400, detail="prompt must be a string or a list of token ids")

    def _text(ids):
        return tokenizer.decode(ids) if tokenizer is not None else None

    @app.get("/health")
    def health():
        eng = loop.engine
        return {"status": "error" if loop.error else "ok", "phase": getattr(eng, "phase", "idle"),
                "error": loop.error, "running": len(eng.sched.running), "waiting": len(eng.sched.waiting)}

    @app.get("/metrics")
    def metrics():
        m = getattr(loop.engine, "metrics", None)
        return PlainTextResponse(m.render() if m is not None else "", media_type="text/plain; version=0.0.4")

    @app.get("/v1/models")
    def models(authorization: str | None = Header(default=None)):
        _auth(authorization)
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "rocket_b200"}]}

    @app.post("/v1/completions")
    async def completions(body: dict, authorization: str | None = Header(default=None)):
        _auth(authorization)
        _greedy_only(body)
        ids = _prompt_ids(body)
        stop = tuple(int(x) for x in body.get("stop_token_ids", []) or [])
        return await _serve(body, ids, stop, chat=False)

    @app.post("/v1/chat/completions")
    async def chat_completions(body: dict, authorization: str | None = Header(default=None)):
        _auth(authorization)
        _greedy_only(body)
        if tokenizer is None:
            raise HTTPException(status_code=400, detail="chat needs a tokenizer (--tokenizer)")
        msgs = body.get("messages")
        if not isinstance(msgs, list) or not msgs or not all(
                isinstance(m, dict) and isinstance(m.get("role"), str) and isinstance(m.get("content"), str)
                for m in msgs):
            raise HTTPException(status_code=400, detail="messages must be a non-empty list of {role, content}")
        ids = tokenizer.encode(render_chat(msgs, chat_template))  # special tokens of the template are kept
        stop = tuple(int(x) for x in body.get("stop_token_ids", []) or []) + tuple(eos_ids)
        return await _serve(body, ids, stop, chat=True)

    def _greedy_only(body):
        if float(body.get("temperature", 0.0) or 0.0) != 0.0 or float(body.get("top_p", 1.0) or 1.0) != 1.0:
            raise HTTPException(status_code=400, detail="only greedy decoding is served (temperature 0, top_p 1)")

    async def _serve(body, ids, stop, chat: bool):
        n = int(body.get("max_tokens", body.get("max_completion_tokens", 16)))
        if not 1 <= n <= max_tokens_limit:
            raise HTTPException(status_code=400, detail=f"max_tokens must be in [1, {max_tokens_limit}]")
        try:
            p = loop.submit(ids, n, stop, asyncio.get_running_loop())
        except QueueFull as e:
            raise HTTPException(status_code=429, detail=str(e), headers={"Retry-After": "1"})
        except (RuntimeError, ValueError) as e:
            raise HTTPException(status_code=503 if loop.error else 400, detail=str(e))
        cid = f"{'chatcmpl' if chat else 'cmpl'}-{next(_ids)}"
        created = int(time.time())
        obj = "chat.completion" if chat else "text_completion"

        def choice(new_ids, text, finish, final=False):
            if not chat:
                c = {"index": 0, "token_ids": new_ids, "finish_reason": finish}
                if text is not None:
                    c["text"] = text
                return c
            if final:
                return {"index": 0, "message": {"role": "assistant", "content": text}, "token_ids": new_ids,
                        "finish_reason": finish}
            return {"index": 0, "delta": {"content": text or ""}, "token_ids": new_ids, "finish_reason": finish}

        async def tokens():
            while True:
                item = await p.queue.get()
                if isinstance(item, Exception):
                    raise item
                if item is None:
                    return
                yield item

        if body.get("stream"):
            chunk_obj = "chat.completion.chunk" if chat else obj

            async def sse():
                done_ids: list[int] = []
                emitted = 0  # characters of the decoded text already sent
                complete = False
                try:
                    if chat:  # the role opens an OpenAI chat stream
                        yield "data: " + json.dumps({"id": cid, "object": chunk_obj, "created": created,
                                                     "model": model_name, "choices": [
                                                         {"index": 0, "delta": {"role": "assistant"},
                                                          "finish_reason": None}]}) + "\n\n"
                    async for new in tokens():
                        text = None
                        if tokenizer is not None:
                            # decode the whole output and send the new suffix, holding back a
                            # trailing replacement character (a UTF-8 sequence split across tokens)
                            done_ids += new
                            full = _text(_visible(done_ids, stop if chat else ()))
                            stable = len(full.rstrip("\ufffd"))
                            text = full[emitted:stable]
                            emitted = max(emitted, stable)
                        yield "data: " + json.dumps({"id": cid, "object": chunk_obj, "created": created,
                                                     "model": model_name, "choices": [choice(new, text, None)]}) + "\n\n"
                    tail = _text(_visible(done_ids, stop if chat else ()))[emitted:] if tokenizer is not None else None
                    yield "data: " + json.dumps({"id": cid, "object": chunk_obj, "created": created,
                                                 "model": model_name, "choices": [choice([], tail, _finish(p))]}) + "\n\n"
                    yield "data: [DONE]\n\n"
                    complete = True
                except Exception as e:  # engine fault mid-stream
                    complete = True
                    yield "data: " + json.dumps({"error": str(e)}) + "\n\n"
                finally:
                    if not complete:  # the client went away: stop generating for it
                        loop.cancel(p)
            return StreamingResponse(sse(), media_type="text/event-stream")

        out: list[int] = []
        try:
            async for new in tokens():
                out += new
        except Exception as e:
            return JSONResponse(status_code=503, content={"error": str(e)})
        text = _text(_visible(out, stop if chat else ())) if tokenizer is not None else None
        r = p.req
        timing = {}
        if r is not None and r.t_first is not None:
            timing = {"ttft_ms": round((r.t_first - r.arrival) * 1e3, 3),
                      "total_ms": round(((r.t_done or time.perf_counter()) - r.arrival) * 1e3, 3)}
        return {"id": cid, "object": obj, "created": created, "model": model_name,
                "choices": [choice(out, text, _finish(p), final=True)],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": len(out),
                          "total_tokens": len(ids) + len(out)}, "timing": timing}

    return app


DEFAULT_CHAT_TEMPLATE = ("{% for m in messages %}<|{{ m['role'] }}|>\n{{ m['content'] }}\n{% endfor %}"
                         "{% if add_generation_prompt %}<|assistant|>\n{% endif %}")


def render_chat(messages: list, template: str | None = None) -> str:
    """Chat messages -> prompt text through a Jinja chat template (sandboxed)."""
    from jinja2.sandbox import ImmutableSandboxedEnvironment
    env = ImmutableSandboxedEnvironment(trim_blocks=False, lstrip_blocks=False)
    return env.from_string(template or DEFAULT_CHAT_TEMPLATE).render(messages=messages, add_generation_prompt=True)


def chat_config(tokenizer_json: str) -> tuple[str | None, list[str]]:
    """(chat template, eos token strings) from the tokenizer_config.json next to a
    tokenizer.json (None, [] if absent)."""
    import os
    p = os.path.join(os.path.dirname(os.path.abspath(tokenizer_json)), "tokenizer_config.json")
    if not os.path.exists(p):
        return None, []
    with open(p) as f:
        cfg = json.load(f)
    tpl = cfg.get("chat_template")
    if isinstance(tpl, list):  # named templates: take the default one
        tpl = next((t.get("template") for t in tpl if t.get("name") == "default"), None)
    eos = cfg.get("eos_token")
    eos = eos.get("content") if isinstance(eos, dict) else eos
    return tpl, [eos] if eos else []


def _visible(ids: list, stop: tuple) -> list:
    """A chat reply without its terminating stop token."""
    return ids[:-1] if ids and stop and ids[-1] in stop else ids


def _finish(p: _Pending) -> str:
    r = p.req
    if r is not None and r.output and r.output[-1] in p.stop:
        return "stop"
    return "length"
