"""Adaptive speculation depth (engine/depth.py): simulated steps with known per-position
acceptance rates and step costs; the policy must settle on the depth that maximises
expected tokens per millisecond, and stay there (exploration aside)."""
import random

import pytest

from rocket_b200.engine.depth import DepthPolicy


def _simulate(rates, steps=600, batch=16, seed=0, base=10.0, per_draft=0.75):
    rng = random.Random(seed)
    K = len(rates)
    pol = DepthPolicy(K)
    prev = K  # drafts available to the first verify
    depths = []
    for _ in range(steps):
        d = pol.decide()
        acc = []
        for _ in range(batch):
            a = 0
            while a < prev and rng.random() < rates[a]:
                a += 1
            acc.append(a)
        ms = base + per_draft * prev + per_draft * d  # verify width and draft passes both cost
        pol.observe(prev, d, acc, ms)
        prev = d
        depths.append(d)
    return pol, depths


def _optimum(rates, base=10.0, per_draft=0.75):
    best, arg = 0.0, 0
    for d in range(len(rates) + 1):
        e, p = 1.0, 1.0
        for j in range(d):
            p *= rates[j]
            e += p
        t = e / (base + 2 * per_draft * d)
        if t > best:
            best, arg = t, d
    return arg


@pytest.mark.parametrize("rates", [[0.9, 0.8, 0.7], [0.3, 0.2, 0.1], [0.0, 0.0, 0.0], [0.8, 0.1, 0.1]])
def test_policy_settles_on_the_best_depth(rates):
    pol, depths = _simulate(rates)
    want = _optimum(rates)
    assert pol.depth == want, (pol.summary(), want)
    tail = depths[-128:]
    # the regime depth, except the periodic exploration step at depth K
    assert sum(d == want for d in tail) >= len(tail) - 3, tail


def test_probes_cycle_and_exploration_reaches_depth_k():
    pol = DepthPolicy(3, explore_every=16)
    first = [pol.decide() for _ in range(16)]
    assert first == [0, 0, 1, 1, 2, 2, 3, 3] * 2  # each depth twice in a row: steady-state costs
    pol.cost = {0: 10.0}
    pol.depth = 0
    seen = [pol.decide() for _ in range(40)]
    assert 3 in seen  # exploration


def test_acceptance_bookkeeping():
    pol = DepthPolicy(3)
    pol.observe(3, 3, [0, 1, 3, 2], 12.0)
    # position 1 checked 4 times, accepted 3; position 2 checked 3 times (a >= 1), accepted 2; ...
    assert pol.tried[1:] == [4, 3, 2] and pol.accepted[1:] == [3, 2, 1]
    assert pol.cost == {3: 12.0}
    pol.observe(2, 3, [2], 11.0)  # a transition step: no cost sample
    assert pol.cost == {3: 12.0}
