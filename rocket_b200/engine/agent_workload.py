"""Forked-prefix agent workloads: a seeded event trace, its causality check and
KV-sharing summary, and a replay driver over any completion backend.

Load shape (agent / sub-agent serving): one root session prefills a long shared
prefix; planner sessions fork from it; an active session below the depth limit
now and then forks a burst of 2-5 children that inherit its whole context (the
fork point) and add a short divergent prefill of their own; tool results land as
mid-stream prefill bursts every few dozen decoded tokens; some sessions go idle
once and resume.  Each tick serves up to ``concurrency`` sessions, least recently
served first, each decoding 8-32 tokens.

Events (dicts; every event has ``t`` = tick and ``seq`` = emission order)::

    session_start {session, parent_id, depth, fork_point_tokens}
    prefill       {session, n_tokens, kind: root | fork | tool}
    decode        {session, n_tokens}
    idle          {session, seconds}
    resume        {session}
    session_end   {session}

The event names and fields follow the reference's trace format so traces are
interchangeable (scripts/scheduler/agent-workload.py:1-24, README.md there);
``session_end`` is this build's addition.  The generator, summary and replay are
this build's own; the per-token KV cost comes from the model config
(``kv_bytes_per_token``) instead of a fuel YAML.

Replay: a session's history is a token list.  ``prefill`` appends random ids,
a fork copies the parent's history, and every ``decode`` becomes a completion
request whose prompt is the session's whole history (so a prefix cache sees the
shared prefix and everything before the session's last turn).  A tick's requests
run concurrently; the generated tokens are appended to the history.
"""
from __future__ import annotations

import json
import random
import time
from dataclasses import dataclass, field


@dataclass
class _Sess:
    sid: str
    parent: str | None
    depth: int
    ctx: int
    fork_point: int
    end_tick: int
    last_served: int = -1
    next_tool: int = 0
    since_tool: int = 0
    idle_at: int | None = None
    idle_until: int | None = None
    idled: bool = False
    children: list = field(default_factory=list)


def agent_trace(concurrency: int = 16, depth: int = 2, prefix_tokens: int = 8192, tool_burst_tokens: int = 300,
                duration_steps: int = 2000, seed: int = 0, fork_prob: float = 0.03, idle_frac: float = 0.2,
                tick_s: float = 1.0, max_context: int | None = None) -> list[dict]:
    """Generate a forked-prefix agent trace (see the module docstring).
    `max_context` ends a session whose context would pass it (engine limit)."""
    if concurrency < 1 or depth < 1 or prefix_tokens < 1 or duration_steps < 1:
        raise ValueError("concurrency, depth, prefix_tokens and duration_steps must be >= 1")
    rng = random.Random(seed)
    ev: list[dict] = []

    def emit(t, event, **kw):
        ev.append({"t": t, "seq": len(ev), "event": event, **kw})

    sess: dict[str, _Sess] = {}
    live: list[str] = []
    nid = [0]

    def start(t, parent: _Sess | None, lifetime: int, kind: str, n_pre: int) -> _Sess | None:
        if parent is not None and max_context is not None and parent.ctx + n_pre > max_context:
            return None  # the fork would not fit the engine's context
        sid = f"s{nid[0]}"
        nid[0] += 1
        fp = parent.ctx if parent else 0
        s = _Sess(sid, parent.sid if parent else None, parent.depth + 1 if parent else 0, fp, fp,
                  t + max(1, lifetime))
        s.next_tool = rng.randint(20, 80)
        if parent is not None and rng.random() < idle_frac:
            s.idle_at = t + rng.randint(1, max(1, lifetime - 1))
        sess[sid] = s
        emit(t, "session_start", session=sid, parent_id=s.parent, depth=s.depth, fork_point_tokens=fp)
        emit(t, "prefill", session=sid, n_tokens=n_pre, kind=kind)
        s.ctx += n_pre
        if parent is not None:
            parent.children.append(sid)
        live.append(sid)
        return s

    def end(t, s: _Sess):
        emit(t, "session_end", session=s.sid)
        live.remove(s.sid)

    root = start(0, None, duration_steps + 1, "root", prefix_tokens)
    n_planners = max(1, concurrency // 2)
    for _ in range(n_planners):
        start(0, root, rng.randint(duration_steps // 4 + 1, duration_steps), "fork", rng.randint(50, 200))
    for t in range(1, duration_steps + 1):
        # lifetimes, idles, resumes
        for sid in list(live):
            s = sess[sid]
            if sid != root.sid and t >= s.end_tick:
                end(t, s)
                continue
            if s.idle_until is not None and t >= s.idle_until:
                s.idle_until = None
                emit(t, "resume", session=sid)
            elif s.idle_at is not None and not s.idled and t >= s.idle_at:
                secs = round(rng.uniform(5.0, 180.0), 1)
                s.idled, s.idle_until = True, t + max(1, int(secs / tick_s))
                emit(t, "idle", session=sid, seconds=secs)
        # keep the planner population (forks of the root) topped up
        planners = [x for x in live if sess[x].parent == root.sid]
        while len(planners) < n_planners:
            p = start(t, root, rng.randint(duration_steps // 8 + 1, duration_steps // 2 + 1), "fork",
                      rng.randint(50, 200))
            if p is None:
                break
            planners.append(p.sid)
        ready = [sess[x] for x in live if x != root.sid and sess[x].idle_until is None]
        ready.sort(key=lambda s: (s.last_served, int(s.sid[1:])))
        served = ready[:concurrency]
        for s in served:
            n = rng.randint(8, 32)
            if max_context is not None and s.ctx + n > max_context:
                end(t, s)
                continue
            s.last_served = t
            emit(t, "decode", session=s.sid, n_tokens=n)
            s.ctx += n
            s.since_tool += n
            if s.since_tool >= s.next_tool:
                nb = max(16, int(rng.gauss(tool_burst_tokens, 0.3 * tool_burst_tokens)))
                if max_context is None or s.ctx + nb <= max_context:
                    emit(t, "prefill", session=s.sid, n_tokens=nb, kind="tool")
                    s.ctx += nb
                s.since_tool, s.next_tool = 0, rng.randint(20, 80)
            if s.depth < depth and rng.random() < fork_prob:
                remaining = max(2, s.end_tick - t)
                for _ in range(rng.randint(2, 5)):
                    start(t, s, rng.randint(1, remaining - 1) if remaining > 2 else 1, "fork",
                          rng.randint(50, 200))
    for sid in list(live):
        end(duration_steps + 1, sess[sid])
    return ev


def validate_trace(events: list[dict]) -> list[str]:
    """Causality errors of a trace (empty = valid): events of a session before its
    start or after its end, a fork whose parent is not live, decreasing ticks or
    sequence numbers, non-positive token counts, resume without idle."""
    errs = []
    live: set = set()
    ended: set = set()
    idle: set = set()
    last_t, last_seq = -1, -1
    for e in events:
        if e.get("event") == "summary":
            continue
        k, sid = e.get("event"), e.get("session")
        if e["t"] < last_t or e["seq"] <= last_seq:
            errs.append(f"seq {e['seq']}: ticks or sequence numbers go backwards")
        last_t, last_seq = e["t"], e["seq"]
        if k == "session_start":
            if sid in live or sid in ended:
                errs.append(f"seq {e['seq']}: {sid} started twice")
            p = e.get("parent_id")
            if p is not None and p not in live:
                errs.append(f"seq {e['seq']}: {sid} forks from {p}, which is not live")
            live.add(sid)
            continue
        if sid not in live:
            errs.append(f"seq {e['seq']}: {k} for {sid}, which is not live")
            continue
        if k in ("prefill", "decode") and int(e.get("n_tokens", 0)) < 1:
            errs.append(f"seq {e['seq']}: {k} with n_tokens < 1")
        if k == "idle":
            idle.add(sid)
        elif k == "resume":
            if sid not in idle:
                errs.append(f"seq {e['seq']}: resume of {sid} without idle")
            idle.discard(sid)
        elif k == "session_end":
            live.discard(sid)
            ended.add(sid)
        elif k in ("prefill", "decode") and sid in idle:
            errs.append(f"seq {e['seq']}: {k} for idle session {sid}")
    return errs


def trace_summary(events: list[dict], kv_bytes_per_token: int = 0, fixed_bytes_per_session: int = 0) -> dict:
    """Token totals, the share of context inherited through forks, peak decoding
    concurrency, and the KV bytes every session would hold with and without
    prefix sharing (fixed per-session state, e.g. a recurrent DeltaNet state, is
    never shareable and is charged to every session either way)."""
    ctx: dict = {}
    fork: dict = {}
    per_tick: dict = {}
    for e in events:
        k = e.get("event")
        if k == "session_start":
            ctx[e["session"]] = e["fork_point_tokens"]
            fork[e["session"]] = e["fork_point_tokens"]
        elif k in ("prefill", "decode"):
            ctx[e["session"]] += e["n_tokens"]
            if k == "decode":
                per_tick[e["t"]] = per_tick.get(e["t"], 0) + 1
    total = sum(ctx.values())
    inherited = sum(fork.values())
    n = len(ctx)
    without = total * kv_bytes_per_token + n * fixed_bytes_per_session
    with_ = (total - inherited) * kv_bytes_per_token + n * fixed_bytes_per_session
    return {"sessions": n, "total_tokens": total, "inherited_tokens": inherited, "fresh_tokens": total - inherited,
            "prefix_shared_fraction": round(inherited / total, 4) if total else 0.0,
            "peak_concurrent_decoding": max(per_tick.values(), default=0),
            "kv_bytes_per_token": kv_bytes_per_token, "fixed_bytes_per_session": fixed_bytes_per_session,
            "kv_bytes_without_sharing": without, "kv_bytes_with_sharing": with_,
            "kv_sharing_ratio": round(with_ / without, 4) if without else None}


def write_trace(events: list[dict], path_or_file, summary: dict | None = None):
    f = open(path_or_file, "w") if isinstance(path_or_file, str) else path_or_file
    try:
        for e in events:
            f.write(json.dumps(e) + "\n")
        if summary is not None:
            f.write(json.dumps({"event": "summary", **summary}) + "\n")
    finally:
        if isinstance(path_or_file, str):
            f.close()


def read_trace(path: str) -> list[dict]:
    with open(path) as f:
        return [json.loads(ln) for ln in f if ln.strip()]


# ---------------------------------------------------------------------- replay
@dataclass
class Completion:
    tokens: list
    t_submit: float
    t_first: float | None
    t_tokens: list
    cached: int = 0


class EngineBackend:
    """Runs a tick's requests together on an in-process engine (continuous batching)."""

    def __init__(self, engine):
        self.engine = engine

    def run_batch(self, jobs: list[tuple[list, int]]) -> list[Completion]:
        t0 = time.perf_counter()
        reqs = [self.engine.add_request(p, n) for p, n in jobs]
        while any(r.t_done is None for r in reqs):
            self.engine.step()
        return [Completion(list(r.output), t0, r.t_first, list(r.t_tokens), r.cached) for r in reqs]


def replay_trace(backend, events: list[dict], vocab: int, seed: int = 0, max_ticks: int | None = None,
                 time_limit_s: float | None = None) -> dict:
    """Replay a trace through `backend.run_batch`: a tick's decodes run as one batch.
    An event that depends on a decode of the same tick (the session's tool prefill
    after it, a fork of the session, its end) waits until the batch has returned, so
    every history equals the trace's context.  Returns throughput, latency
    percentiles and how much prompt came from cache."""
    rng = random.Random(seed)
    hist: dict[str, list] = {}
    by_tick: dict[int, list] = {}
    for e in events:
        if e.get("event") != "summary":
            by_tick.setdefault(e["t"], []).append(e)
    comps: list[Completion] = []
    prompt_tok = [0]
    batches = [0]

    def apply(e, jobs, owners):
        k, sid = e["event"], e.get("session")
        if k == "session_start":
            p = e.get("parent_id")
            hist[sid] = list(hist[p]) if p is not None else []
        elif k == "prefill":
            hist[sid] += [rng.randrange(vocab) for _ in range(e["n_tokens"])]
        elif k == "decode":
            jobs.append((list(hist[sid]), e["n_tokens"]))
            owners.append(sid)
        elif k == "session_end":
            hist.pop(sid, None)

    def flush(jobs, owners, deferred):
        if jobs:
            batches[0] += 1
            out = backend.run_batch(jobs)
            for sid, (p, _), c in zip(owners, jobs, out):
                prompt_tok[0] += len(p)
                comps.append(c)
                if sid in hist:
                    hist[sid] += c.tokens
        jobs.clear()
        owners.clear()
        for e in deferred:
            apply(e, jobs, owners)  # no decodes here: a dependent decode flushes first
        deferred.clear()

    t0 = time.perf_counter()
    ticks = 0
    for t in sorted(by_tick):
        if max_ticks is not None and ticks >= max_ticks:
            break
        if time_limit_s is not None and time.perf_counter() - t0 > time_limit_s:
            break
        jobs, owners, deferred = [], [], []
        waiting: set = set()
        for e in by_tick[t]:
            sid = e.get("session")
            touches = {sid, e.get("parent_id")} if e["event"] == "session_start" else {sid}
            if touches & (set(owners) | waiting):
                if e["event"] == "decode":
                    flush(jobs, owners, deferred)
                    waiting.clear()
                else:
                    deferred.append(e)
                    waiting.add(sid)
                    continue
            apply(e, jobs, owners)
        if jobs or deferred:
            ticks += 1 if jobs else 0
            flush(jobs, owners, deferred)
    wall = time.perf_counter() - t0
    out_tok = sum(len(c.tokens) for c in comps)
    ttft = [(c.t_first - c.t_submit) * 1e3 for c in comps if c.t_first]
    itl = []
    for c in comps:
        itl += [(b - a) * 1e3 for a, b in zip(c.t_tokens, c.t_tokens[1:])]
    cached = sum(c.cached for c in comps)
    ptok = prompt_tok[0]

    def pct(a, q):
        a = sorted(a)
        return round(a[min(len(a) - 1, int(q * len(a)))], 3) if a else None

    return {"ticks": ticks, "batches": batches[0], "requests": len(comps), "wall_s": round(wall, 3),
            "output_tokens": out_tok, "output_tok_s": round(out_tok / wall, 2) if wall else None,
            "prompt_tokens": ptok, "cached_prompt_tokens": cached,
            "prompt_cache_fraction": round(cached / ptok, 4) if ptok else 0.0,
            "ttft_ms_p50": pct(ttft, 0.5), "ttft_ms_p95": pct(ttft, 0.95),
            "itl_ms_p50": pct(itl, 0.5), "itl_ms_p95": pct(itl, 0.95)}


def kv_costs(cfg, kv_dtype: str = "bf16") -> tuple[int, int]:
    """(KV bytes per context token, fixed recurrent-state bytes per session) of a whole
    model (all ranks): K + V (or the MLA latent) and the DSA index keys + gates of
    every attention layer; the fp32 DeltaNet state plus conv taps of every linear
    attention layer."""
    eb = 1 if kv_dtype == "fp8" else 2
    n_attn = sum(1 for i in range(cfg.num_layers) if cfg.layer_kind(i) == "attention")
    n_lin = cfg.num_layers - n_attn
    if cfg.mla is not None:
        per_tok = n_attn * cfg.mla.kv_lora_rank * 2
    else:
        per_tok = n_attn * 2 * cfg.num_kv_heads * cfg.head_dim * eb
    if cfg.sparse_attention is not None:
        per_tok += n_attn * 2 * cfg.sparse_attention.index_dim * 2
    fixed = 0
    if n_lin and cfg.deltanet is not None:
        dn = cfg.deltanet
        conv_ch = (2 * dn.num_qk_heads + dn.num_v_heads) * dn.head_dim
        fixed = n_lin * (dn.num_v_heads * dn.head_dim * dn.head_dim * 4 + (dn.conv_kernel - 1) * conv_ch * 2)
    return per_tok, fixed
