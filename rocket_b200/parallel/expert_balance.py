"""Expert-parallel placement from firing histograms.

    order = balance(hist, ranks)                     # native greedy LPT (C++)
    engine = LLMEngine.from_fuel(..., expert_order=order)

``order`` lists experts grouped by owner: rank r serves order[r*E/R:(r+1)*E/R].
The model applies it by permuting router rows (and the sigmoid-routing bias) and
loading those experts' weights, which leaves the model function unchanged.
Histograms come from ``utils.telemetry.Telemetry.fire_histogram()`` and are
stored as JSON.

Counterpart of the reference's expert_balance / load_expert_histogram
(engines/glm5-moe-nvfp4-2b/src/fabric/expert_balance.h:37-53).
"""
from __future__ import annotations

import json


def balance(hist, ranks: int) -> list[int]:
    from .. import _rt
    _, order, _ = _rt.balance_experts([int(x) for x in hist], int(ranks))
    return list(order)


def placement(hist, ranks: int) -> dict:
    from .. import _rt
    owner, order, load = _rt.balance_experts([int(x) for x in hist], int(ranks))
    return {"owner": list(owner), "order": list(order), "rank_load": list(load)}


def contiguous_load(hist, ranks: int) -> list[int]:
    """Per-rank load of the default placement (expert e on rank e // (E/R))."""
    E = len(hist)
    c = E // ranks
    return [int(sum(hist[r * c:(r + 1) * c])) for r in range(ranks)]


def save_histogram(hist, path: str):
    with open(path, "w") as f:
        json.dump({"expert_fires": [int(x) for x in hist]}, f)


def load_histogram(path: str) -> list[int]:
    with open(path) as f:
        return [int(x) for x in json.load(f)["expert_fires"]]
