"""Adaptive speculation depth: how many MTP drafts each engine step produces (and so how
many the next step verifies).

Every depth d in 0..K has its own CUDA graphs (per batch bucket), so a step costs what
its depth needs: d - 1 chained MTP passes after the first, d draft rows verified per
sequence.  The policy picks d to maximise expected emitted tokens per unit of step time:

  E(d) = 1 + sum_{i <= d} prod_{j <= i} p_j        p_j = P(draft j accepted | 1..j-1 were)
  T(d) = E(d) / cost(d)                             cost(d): measured step time at depth d

The acceptance of draft position j is a binomial rate observed only when a step
verified at least j drafts and accepted the first j - 1, so estimates carry Wilson
score bounds (wilson_bounds in drafts.py).  Decisions:

  * probe: the first `probes` steps cycle through depths 0..K, each on two consecutive
    steps (the second one verifies what the first drafted: a steady-state cost sample);
  * explore: every `explore_every` steps draft at depth K once, so deep positions keep
    being observed while a shallow depth is in use;
  * promote: at the end of each `window` of steps, move to the depth with the best
    point estimate when even its lower-bound throughput (Wilson lower bounds of the
    rates) beats the current depth's point estimate by `margin`;
  * demote: move there when the current depth's optimistic throughput (upper bounds)
    stays below the best point estimate for `fail_windows` consecutive windows.

Depth 0 verifies nothing and runs only the MTP block (its KV stays coherent for later
drafting) without the vocabulary head.

Counterpart of the reference's adaptive MTP policy and depth-bucket planner
(engines/qwen38-flash-next-nvfp4-2b/src/qwen38_slab/mtp_policy.py:1-57,413;
qwen38_slab/decode.py:124): the same control ideas (initial probes, Wilson-bound
promotion with a margin, demotion after failing windows, periodic exploration, K0..K7
graph buckets); the throughput model and the state layout here are this engine's own.
"""
from __future__ import annotations

from .drafts import wilson_bounds


class DepthPolicy:
    def __init__(self, K: int, probes: int | None = None, margin: float = 0.03, window: int = 8, fail_windows: int = 2,
                 explore_every: int = 64, z: float = 1.96, ema: float = 0.2):
        if K < 1:
            raise ValueError("adaptive depth needs spec_tokens >= 1")
        self.K = K
        probes = 4 * (K + 1) if probes is None else probes  # two visits of every depth
        self.probes, self.margin, self.window = probes, margin, window
        self.fail_windows, self.explore_every, self.z, self.ema = fail_windows, explore_every, z, ema
        self.tried = [0] * (K + 1)     # [j]: steps x sequences in which draft j was checked
        self.accepted = [0] * (K + 1)  # [j]: ... and accepted
        self.cost: dict[int, float] = {}  # depth -> EMA of the step time (ms) in steady state
        self.depth = K                 # depth of the current regime
        self.decisions = 0
        self.failing = 0
        self.switches = 0
        self.last = K                  # depth drafted by the previous step (= drafts available now)

    # ------------------------------------------------------------------ observations
    def observe(self, verified: int, drafted: int, accepted: list[int], step_ms: float | None):
        """One step: `verified` drafts fed per verify sequence, `drafted` MTP passes run,
        `accepted[i]` drafts accepted by verify sequence i, and the step's time."""
        for a in accepted:
            a = min(a, verified)
            for j in range(1, a + 1):
                self.tried[j] += 1
                self.accepted[j] += 1
            if a < verified:
                self.tried[a + 1] += 1
        if step_ms is not None and verified == drafted:  # steady-state step of depth `drafted`
            c = self.cost.get(drafted)
            self.cost[drafted] = step_ms if c is None else (1 - self.ema) * c + self.ema * step_ms

    # ------------------------------------------------------------------ estimates
    def rate(self, j: int, which: str = "mid") -> float:
        n, k = self.tried[j], self.accepted[j]
        if n == 0:
            return {"lo": 0.0, "mid": 0.5, "hi": 1.0}[which]
        if which == "mid":
            return k / n
        lo, hi = wilson_bounds(k, n, self.z)
        return lo if which == "lo" else hi

    def expected_tokens(self, d: int, which: str = "mid") -> float:
        e, p = 1.0, 1.0
        for j in range(1, d + 1):
            p *= self.rate(j, which)
            e += p
        return e

    def throughput(self, d: int, which: str = "mid") -> float | None:
        c = self.cost.get(d)
        return None if not c else self.expected_tokens(d, which) / c

    def best(self) -> int | None:
        cand = [(self.throughput(d), d) for d in range(self.K + 1) if self.cost.get(d)]
        return max(cand)[1] if cand else None

    # ------------------------------------------------------------------ decision
    def decide(self) -> int:
        """Depth (MTP draft passes) of the next step."""
        i = self.decisions
        self.decisions += 1
        if i < self.probes:
            d = (i // 2) % (self.K + 1)
        elif self.explore_every and i % self.explore_every == 0:
            d = self.K
        else:
            if i % self.window == 0:
                self._review()
            d = self.depth
        self.last = d
        return d

    def _review(self):
        b = self.best()
        cur = self.depth
        if b is None or b == cur or self.throughput(cur) is None:
            self.failing = 0
            if b is not None and self.throughput(cur) is None:
                self.depth = b
            return
        t_cur = self.throughput(cur)
        if self.throughput(b, "lo") > (1 + self.margin) * t_cur:
            self.depth, self.failing = b, 0
            self.switches += 1
            return
        if self.throughput(cur, "hi") < self.throughput(b):
            self.failing += 1
            if self.failing >= self.fail_windows:
                self.depth, self.failing = b, 0
                self.switches += 1
        else:
            self.failing = 0

    def summary(self) -> dict:
        return {"depth": self.depth, "decisions": self.decisions, "switches": self.switches,
                "rates": [round(self.rate(j), 4) for j in range(1, self.K + 1)],
                "tried": self.tried[1:], "cost_ms": {d: round(c, 3) for d, c in sorted(self.cost.items())}}
