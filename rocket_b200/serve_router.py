"""Data-parallel serving: one HTTP endpoint in front of several engine groups.

    # two EP4 engine groups on one 8-GPU box, one endpoint
    CUDA_VISIBLE_DEVICES=0,1,2,3 torchrun --nproc-per-node 4 --master-port 29500 -m rocket_b200 serve --port 8001
    CUDA_VISIBLE_DEVICES=4,5,6,7 torchrun --nproc-per-node 4 --master-port 29501 -m rocket_b200 serve --port 8002
    python -m rocket_b200 route --backend http://127.0.0.1:8001 --backend http://127.0.0.1:8002 --port 8000

Each completion goes to the backend with the fewest requests in flight (ties to the
one that served fewest), so long generations do not pile up behind each other; streams are passed
through chunk by chunk.  A backend that fails a request with a connection error or a 5xx
is marked down for `cooldown_s` and the request is retried on another backend (only
before any byte was sent to the client).  /health reports every backend; /metrics
concatenates the backends' Prometheus text with a `backend` label.

The reference names this arrangement ("replicated" engines, blog/rocket.qmd:83-87) but
does not implement it; here it is a host-side router over independent `serve` processes.
"""
import time  # no postponed annotations here: FastAPI resolves the handlers' parameter types


class Backend:
    def __init__(self, name: str, client):
        self.name = name
        self.client = client     # httpx.AsyncClient with the backend's base URL
        self.inflight = 0
        self.down_until = 0.0
        self.served = 0
        self.failed = 0

    def up(self) -> bool:
        return time.monotonic() >= self.down_until


def pick(backends: list[Backend], exclude=()) -> Backend | None:
    """Least requests in flight among the backends that are up; ties go to the backend that
    served the fewest requests, then the lowest index (round-robin under light load)."""
    best = None
    for b in backends:
        if b in exclude or not b.up():
            continue
        if best is None or (b.inflight, b.served) < (best.inflight, best.served):
            best = b
    return best


def build_router(backends: list[Backend], cooldown_s: float = 5.0, api_key: str | None = None):
    import httpx
    from fastapi import FastAPI, Header, HTTPException, Request
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    app = FastAPI(title="rocket_b200 router")

    def _auth(authorization):
        if api_key and authorization != f"Bearer {api_key}":
            raise HTTPException(status_code=401, detail="bad or missing API key")

    def _headers(authorization):
        return {"Authorization": authorization} if authorization else {}

    @app.get("/health")
    async def health():
        out = []
        for b in backends:
            try:
                r = await b.client.get("/health", timeout=5.0)
                st = r.json()
            except (httpx.HTTPError, ValueError) as e:
                st = {"status": "unreachable", "error": type(e).__name__}
            out.append({"backend": b.name, "inflight": b.inflight, "served": b.served, "failed": b.failed,
                        "up": b.up(), **st})
        ok = any(o.get("status") == "ok" for o in out)
        return JSONResponse(status_code=200 if ok else 503, content={"status": "ok" if ok else "error",
                                                                     "backends": out})

    @app.get("/metrics")
    async def metrics():
        lines = []
        for b in backends:
            try:
                txt = (await b.client.get("/metrics", timeout=5.0)).text
            except httpx.HTTPError:
                continue
            for ln in txt.splitlines():
                if not ln or ln.startswith("#"):
                    lines.append(ln)
                    continue
                name, _, rest = ln.partition(" ")
                if "{" in name:
                    name = name.replace("{", '{backend="%s",' % b.name, 1)
                else:
                    name = name + '{backend="%s"}' % b.name
                lines.append(f"{name} {rest}")
        return PlainTextResponse("\n".join(lines) + "\n", media_type="text/plain; version=0.0.4")

    @app.post("/v1/completions")
    async def completions(request: Request, authorization: str | None = Header(default=None)):
        return await _forward("/v1/completions", request, authorization)

    @app.post("/v1/chat/completions")
    async def chat_completions(request: Request, authorization: str | None = Header(default=None)):
        return await _forward("/v1/chat/completions", request, authorization)

    async def _forward(path: str, request, authorization):
        _auth(authorization)
        body = await request.json()
        tried = []
        while True:
            b = pick(backends, tried)
            if b is None:
                raise HTTPException(status_code=503, detail="no engine group available")
            tried.append(b)
            b.inflight += 1
            if body.get("stream"):
                try:
                    req = b.client.build_request("POST", path, json=body, headers=_headers(authorization),
                                                 timeout=None)
                    resp = await b.client.send(req, stream=True)
                except httpx.HTTPError:
                    b.inflight -= 1
                    b.failed += 1
                    b.down_until = time.monotonic() + cooldown_s
                    continue
                if resp.status_code >= 500:
                    await resp.aclose()
                    b.inflight -= 1
                    b.failed += 1
                    b.down_until = time.monotonic() + cooldown_s
                    continue

                async def relay(resp=resp, b=b):
                    try:
                        async for chunk in resp.aiter_raw():
                            yield chunk
                    finally:
                        await resp.aclose()
                        b.inflight -= 1
                        b.served += 1
                return StreamingResponse(relay(), status_code=resp.status_code,
                                         media_type=resp.headers.get("content-type", "text/event-stream"))
            try:
                r = await b.client.post(path, json=body, headers=_headers(authorization), timeout=None)
            except httpx.HTTPError:
                b.failed += 1
                b.down_until = time.monotonic() + cooldown_s
                continue
            finally:
                b.inflight -= 1
            if r.status_code >= 500:
                b.failed += 1
                b.down_until = time.monotonic() + cooldown_s
                continue
            b.served += 1
            return JSONResponse(status_code=r.status_code, content=r.json())

    return app


def backends_from_urls(urls: list[str]) -> list[Backend]:
    import httpx
    return [Backend(u, httpx.AsyncClient(base_url=u)) for u in urls]
