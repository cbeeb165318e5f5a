"""Quality gates: a deterministic task set with long-context needle retrieval, run over
an OpenAI-style completions endpoint, and teacher-forced perplexity of a text.

    python -m rocket_b200 quality --url http://127.0.0.1:8000 --out q.json [--compare base.json]
    python -m rocket_b200 perplexity --fuel F --fuel-dir D --tokenizer tokenizer.json --text-file wiki.txt

``quality`` sends every task greedily (temperature 0) and grades the lower-cased
completion (reasoning blocks stripped; see ``grade``); ``--compare`` fails (exit 1)
on any task that passed in the baseline
report and fails now -- the gate a quantization or kernel change must clear.
``perplexity`` scores the text in windows with ``LLMEngine.teacher_nll``.

Counterparts of the reference's numerics gates (scripts/numerics/qwen38-quality.py:
deterministic cases + needles, regression compare; WikiText perplexity in its
numerics notes).  The task set and the needle text here are this build's own.
"""
from __future__ import annotations

import json
import math
import re
import time

TASKS = [
    ("arith", "Work it out: (36 * 25 - 150) / 6 + 13. Finish with the number alone.", ["138"]),
    ("percent", "A jacket costs 80 dollars. It is discounted by 25 percent, and then 10 dollars of tax is "
                "added. What is the final price in dollars? Give only the number.", ["70"]),
    ("weekday", "Today is Monday. Which day of the week will it be 45 days from today? One word.", ["thursday"]),
    ("modpow", "Compute 3^50 mod 7. Give one integer.", ["2"]),
    ("letters", "How many times does the letter 'e' occur in 'excellence'? Give one integer.", ["4"]),
    ("sort", "List these numbers from largest to smallest, comma separated, nothing else: 0.5, 0.45, 0.054, "
             "0.505.", ["0.505, 0.5, 0.45, 0.054"]),
    ("syllogism", "All wugs are daxes. No daxes are feps. Can a wug be a fep? Answer yes or no first.", ["no"]),
    ("rates", "Two pipes fill a pool: one alone takes 6 hours, the other alone takes 3 hours. How many hours "
              "do they take together? Give one number.", ["2"]),
    ("who", "Dana is taller than Eli. Eli is taller than Fay. Who is the shortest? One name.", ["fay"]),
    ("primes", "What is the sum of the prime numbers below 20? Give one integer.", ["77"]),
]

_FILL = "Entry {i:05d}: the harbour office noted that berth {b} was swept and inspected on schedule.\n"


def needle_task(depth_tokens: int, secret: str) -> str:
    """~depth_tokens of filler (about 16 tokens a line) with one line holding `secret`
    at the middle, then the question."""
    rows = [_FILL.format(i=i, b=i % 9 + 1) for i in range(max(1, depth_tokens // 16))]
    mid = len(rows) // 2
    rows.insert(mid, f"Entry {mid:05d}: the vault code for this ledger is {secret}.\n")
    return "".join(rows) + "\nWhat is the vault code for this ledger? Reply with the code only."


def task_set(needles=(8000, 64000)) -> list[tuple[str, str, list[str]]]:
    out = list(TASKS)
    for i, d in enumerate(needles):
        secret = f"AMBER-LANTERN-{4821 + i}"
        out.append((f"needle_{d}", needle_task(int(d), secret), [secret.lower()]))
    return out


_NUM = re.compile(r"-?\d+(?:\.\d+)?")


def grade(text: str, accepted: list[str]) -> bool:
    """Numeric answers must be the completion's last number; single words must appear as
    a whole word; anything else as a substring (reasoning blocks are ignored)."""
    ans = re.sub(r"<think>.*?</think>", " ", text, flags=re.I | re.S).lower()
    nums = _NUM.findall(ans)
    for a in accepted:
        if _NUM.fullmatch(a):
            if nums and float(nums[-1]) == float(a):
                return True
        elif re.fullmatch(r"[a-z]+", a):
            if re.search(rf"\b{a}\b", ans):
                return True
        elif a in ans:
            return True
    return False


def _ask(url: str, prompt: str, max_tokens: int, model: str | None, timeout: float):
    import requests
    body = {"prompt": prompt, "max_tokens": max_tokens, "temperature": 0}
    if model:
        body["model"] = model
    t0 = time.monotonic()
    r = requests.post(url.rstrip("/") + "/v1/completions", json=body, timeout=timeout)
    r.raise_for_status()
    js = r.json()
    return js["choices"][0].get("text") or "", js.get("usage", {}), time.monotonic() - t0


def run_quality(url: str, max_tokens: int = 1024, needles=(8000, 64000), model: str | None = None,
                timeout: float = 900.0, ask=None) -> dict:
    """Run the task set against a server (or `ask(prompt, max_tokens) -> (text, usage, s)`)."""
    ask = ask or (lambda p, n: _ask(url, p, n, model, timeout))
    results = {}
    for name, prompt, accepted in task_set(needles):
        text, usage, secs = ask(prompt, max_tokens)
        results[name] = {"ok": grade(text, accepted), "answer_tail": text.strip()[-160:], "seconds": round(secs, 2),
                         "prompt_tokens": usage.get("prompt_tokens"),
                         "completion_tokens": usage.get("completion_tokens")}
    return {"passed": sum(r["ok"] for r in results.values()), "total": len(results), "results": results}


def regressions(report: dict, baseline: dict) -> list[str]:
    """Tasks that passed in `baseline` and fail in `report`."""
    return sorted(n for n, r in report["results"].items()
                  if baseline.get("results", {}).get(n, {}).get("ok") and not r["ok"])


def perplexity(engine, ids: list[int], window: int = 2048, stride: int | None = None) -> dict:
    """Perplexity of `ids` scored in windows of `window` tokens advancing by `stride`
    (default: non-overlapping); with overlap, only the tokens past the previous
    window's end are counted, each conditioned on up to `window` tokens."""
    stride = stride or window
    if window < 2 or stride < 1 or stride > window:
        raise ValueError("need window >= 2 and 1 <= stride <= window")
    nll_sum, n, end_prev = 0.0, 0, 0
    t0 = time.perf_counter()
    for s0 in range(0, max(1, len(ids) - 1), stride):
        seg = ids[s0:s0 + window]
        if len(seg) < 2:
            break
        nll = engine.teacher_nll(seg)          # nll[i] scores seg[i + 1] = ids[s0 + i + 1]
        first_new = max(0, end_prev - s0 - 1)  # ids up to end_prev were scored already
        take = nll[first_new:]
        nll_sum += sum(take)
        n += len(take)
        end_prev = s0 + len(seg)
        if end_prev >= len(ids):
            break
    wall = time.perf_counter() - t0
    mean = nll_sum / n if n else float("nan")
    return {"tokens_scored": n, "nll_mean": round(mean, 6), "perplexity": round(math.exp(mean), 4) if n else None,
            "window": window, "stride": stride, "wall_s": round(wall, 3),
            "tok_s": round(n / wall, 1) if wall else None}


def write_report(report: dict, path: str):
    with open(path, "w", encoding="utf-8") as f:
        json.dump(report, f, indent=2, sort_keys=True)
