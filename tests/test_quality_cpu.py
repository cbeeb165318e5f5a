"""Quality gates on CPU: grading rules, the task runner with a scripted model,
regression compare, perplexity windowing, and the vocabulary-sharded NLL on gloo ranks
against a full log-softmax."""
import math
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from rocket_b200.quality import grade, perplexity, regressions, run_quality, task_set


def test_grading_rules():
    assert grade("... so the result is 138", ["138"]) and not grade("138, no wait, 139", ["138"])
    assert grade("Thursday.", ["thursday"]) and not grade("Thursdays", ["thursday"])
    assert grade("<think>maybe yes</think> No.", ["no"]) and not grade("<think>no</think> yes", ["no"])
    assert grade("the code is amber-lantern-4821", ["amber-lantern-4821"])
    assert grade("0.505, 0.5, 0.45, 0.054", ["0.505, 0.5, 0.45, 0.054"])


def test_task_answers_are_right():
    """The accepted answers of the arithmetic tasks, recomputed."""
    acc = {n: a for n, _, a in task_set(())}
    assert acc["arith"] == [str((36 * 25 - 150) // 6 + 13)]
    assert acc["percent"] == [str(int(80 * 0.75 + 10))]
    assert acc["modpow"] == [str(pow(3, 50, 7))]
    assert acc["letters"] == [str("excellence".count("e"))]
    assert acc["primes"] == [str(sum(p for p in range(2, 20) if all(p % q for q in range(2, p))))]
    days = ["monday", "tuesday", "wednesday", "thursday", "friday", "saturday", "sunday"]
    assert acc["weekday"] == [days[45 % 7]]
    assert acc["sort"] == [", ".join(str(x) for x in sorted([0.5, 0.45, 0.054, 0.505], reverse=True))]


def test_runner_and_regressions():
    tasks = {p: a for _, p, a in task_set((512,))}

    def oracle(prompt, n):
        return f"Answer: {tasks[prompt][0]}", {"prompt_tokens": len(prompt) // 4, "completion_tokens": 3}, 0.01

    rep = run_quality("unused", 64, (512,), ask=oracle)
    assert rep["passed"] == rep["total"] == len(tasks)
    assert "needle_512" in rep["results"]
    bad = run_quality("unused", 64, (512,), ask=lambda p, n: ("I do not know", {}, 0.0))
    assert bad["passed"] == 0
    assert regressions(bad, rep) == sorted(rep["results"])
    assert regressions(rep, bad) == []


class _NllEngine:
    """teacher_nll(seg)[i] = value of the scored token (ids are their own NLL)."""

    def __init__(self):
        self.calls = []

    def teacher_nll(self, seg):
        self.calls.append(list(seg))
        return [float(x) for x in seg[1:]]


@pytest.mark.parametrize("n,window,stride", [(100, 32, 32), (100, 32, 8), (33, 32, 32), (10, 64, None)])
def test_perplexity_scores_every_token_once(n, window, stride):
    ids = list(range(1, n + 1))
    eng = _NllEngine()
    res = perplexity(eng, ids, window, stride)
    assert all(len(c) <= window for c in eng.calls)
    if stride is None or stride == window:
        # non-overlapping windows: the first token of every window has no context
        scored = [x for c in eng.calls for x in c[1:]]
    else:
        scored = ids[1:]
    assert res["tokens_scored"] == len(scored)
    assert res["nll_mean"] == pytest.approx(sum(scored) / len(scored), rel=1e-6)
    assert res["perplexity"] == pytest.approx(math.exp(sum(scored) / len(scored)), rel=1e-4)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nll_worker(rank, world, port, q):
    import torch.distributed as dist

    from rocket_b200.engine.engine import sharded_token_nll
    from rocket_b200.parallel.context import ParallelCtx
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(0)
    V, R = 50, 7
    lg = torch.randn(R, V, generator=g) * 3
    tgt = torch.randint(0, V, (R,), generator=g)
    cuts = [0, 17, V] if world == 2 else [0, V]
    par = ParallelCtx(rank, world, device="cpu")
    got = sharded_token_nll(lg[:, cuts[rank]:cuts[rank + 1]].contiguous(), tgt, cuts[rank], par)
    ref = -torch.log_softmax(lg, -1).gather(1, tgt[:, None])[:, 0]
    q.put((rank, torch.allclose(got, ref, atol=1e-5, rtol=1e-5)))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2])
def test_sharded_nll_equals_full_log_softmax(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_nll_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    assert all(ok for _, ok in res), res
