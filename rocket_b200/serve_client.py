"""HTTP load generator for any OpenAI-style completions endpoint (this package's
``serve`` / ``route``, or another server taking token-id prompts).

    python -m rocket_b200 http-bench --url http://127.0.0.1:8000 --workload poisson \
        --requests 256 --rate 4 --prompt-lo 1024 --prompt-hi 8192 --mean-out 256
    python -m rocket_b200 http-bench --url http://127.0.0.1:8000 --workload agent \
        --concurrency 16 --duration-steps 200

Every request streams (server-sent events), so time to first token and the gaps
between tokens are measured on the client.  ``poisson`` sends an open-loop Poisson
workload (at most ``--max-inflight`` requests in flight); ``agent`` replays a
forked-prefix agent trace tick by tick (engine/agent_workload.py), which exercises
the server's prefix cache.

Counterpart of the reference's OpenAI-API baseline load generator
(scripts/baseline/openai-forked-prefix.py); the client here is this build's own.
"""
from __future__ import annotations

import json
import threading
import time
from concurrent.futures import ThreadPoolExecutor

from .engine.agent_workload import Completion


def stream_completion(url: str, prompt: list, max_tokens: int, model: str | None = None, api_key: str | None = None,
                      timeout_s: float = 600.0) -> Completion:
    """POST one streaming completion with a token-id prompt; returns the tokens with
    the client-side submit / first-token / per-token times."""
    import requests
    body = {"prompt": list(map(int, prompt)), "max_tokens": int(max_tokens), "stream": True, "temperature": 0}
    if model:
        body["model"] = model
    headers = {"Authorization": f"Bearer {api_key}"} if api_key else {}
    t0 = time.perf_counter()
    toks, times = [], []
    with requests.post(url.rstrip("/") + "/v1/completions", json=body, headers=headers, stream=True,
                       timeout=timeout_s) as r:
        if r.status_code != 200:
            raise RuntimeError(f"completion failed: HTTP {r.status_code}: {r.text[:200]}")
        for ln in r.iter_lines(decode_unicode=True):
            if not ln or not ln.startswith("data: "):
                continue
            data = ln[6:]
            if data == "[DONE]":
                break
            ids = json.loads(data)["choices"][0].get("token_ids") or []
            now = time.perf_counter()
            toks += ids
            times += [now] * len(ids)
    return Completion(toks, t0, times[0] if times else None, times)


class HttpBackend:
    """Runs each batch of (prompt, max_new) jobs concurrently against a server."""

    def __init__(self, url: str, max_inflight: int = 64, model: str | None = None, api_key: str | None = None):
        self.url, self.model, self.api_key = url, model, api_key
        self.pool = ThreadPoolExecutor(max_workers=max_inflight)

    def run_batch(self, jobs):
        futs = [self.pool.submit(stream_completion, self.url, p, n, self.model, self.api_key) for p, n in jobs]
        return [f.result() for f in futs]

    def close(self):
        self.pool.shutdown(wait=True)


def run_http_open_loop(url: str, workload, max_inflight: int = 64, model: str | None = None,
                       api_key: str | None = None) -> dict:
    """Open-loop replay of an `Arrival` workload (engine/loadgen.py) over HTTP."""
    pool = ThreadPoolExecutor(max_workers=max_inflight)
    lock = threading.Lock()
    done: list[Completion] = []
    errors: list[str] = []

    def job(a):
        try:
            c = stream_completion(url, a.prompt, a.max_new_tokens, model, api_key)
            with lock:
                done.append(c)
        except Exception as e:  # recorded, the run continues
            with lock:
                errors.append(str(e)[:200])

    t0 = time.perf_counter()
    futs = []
    for a in sorted(workload, key=lambda a: a.t):
        wait = a.t - (time.perf_counter() - t0)
        if wait > 0:
            time.sleep(wait)
        futs.append(pool.submit(job, a))
    for f in futs:
        f.result()
    pool.shutdown(wait=True)
    wall = time.perf_counter() - t0
    out_tok = sum(len(c.tokens) for c in done)
    ttft = sorted((c.t_first - c.t_submit) * 1e3 for c in done if c.t_first)
    itl = sorted((b - a) * 1e3 for c in done for a, b in zip(c.t_tokens, c.t_tokens[1:]))

    def pct(a, q):
        return round(a[min(len(a) - 1, int(q * len(a)))], 3) if a else None

    return {"requests": len(workload), "completed": len(done), "errors": len(errors),
            "first_error": errors[0] if errors else None, "wall_s": round(wall, 3), "output_tokens": out_tok,
            "output_tok_s": round(out_tok / wall, 2) if wall else None,
            "prompt_tokens": sum(len(a.prompt) for a in workload),
            "ttft_ms_p50": pct(ttft, 0.5), "ttft_ms_p95": pct(ttft, 0.95),
            "itl_ms_p50": pct(itl, 0.5), "itl_ms_p95": pct(itl, 0.95)}
