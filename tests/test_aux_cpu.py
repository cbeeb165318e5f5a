"""Host runtime pieces on the CPU: expert balancing (greedy LPT, equal cardinality,
deterministic) and the Prometheus metrics rendering.

Expert balancing mirrors the reference's expert_balance tests
(engines/glm5-moe-nvfp4-2b/src/fabric/expert_balance.cc:58-102).
"""
import random

from rocket_b200.parallel import expert_balance as eb
from rocket_b200.utils.metrics import Metrics


def test_balance_equal_cardinality_and_better_than_contiguous():
    rnd = random.Random(0)
    E, R = 160, 8
    # skewed: hot experts clustered at low ids (the contiguous split puts them on rank 0)
    hist = [int(1000 * (0.97 ** e) + rnd.randint(0, 20)) for e in range(E)]
    p = eb.placement(hist, R)
    owner, order, load = p["owner"], p["order"], p["rank_load"]
    assert sorted(order) == list(range(E))
    for r in range(R):
        assert sum(1 for o in owner if o == r) == E // R
        assert all(owner[e] == r for e in order[r * E // R:(r + 1) * E // R])
    assert sum(load) == sum(hist)
    contig = eb.contiguous_load(hist, R)
    assert max(load) < max(contig) / 3
    assert max(load) - min(load) <= max(hist)  # LPT bound
    assert eb.balance(hist, R) == order  # deterministic


def test_balance_rejects_bad_shapes():
    import pytest
    with pytest.raises(Exception):
        eb.balance([1, 2, 3], 2)


def test_metrics_render():
    m = Metrics(labels={"rank": 0})
    m.inc("requests_total", 3)
    m.inc("generated_tokens_total", 42)
    m.set("running_requests", 2)
    for v in (3, 7, 40):
        m.observe("step_ms", v)
    txt = m.render()
    assert 'rocket_b200_requests_total{rank="0"} 3' in txt
    assert 'rocket_b200_step_ms_bucket{le="5",rank="0"} 1' in txt
    assert 'rocket_b200_step_ms_count{rank="0"} 3' in txt
    assert "# TYPE rocket_b200_itl_ms histogram" in txt
