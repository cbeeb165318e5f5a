"""Model health telemetry of eager forward passes: per-layer residual RMS, router
entropy, expert fire counts and per-site activation absmax.

    tel = Telemetry(engine.model)
    with tel:                       # hooks installed only inside the block
        engine.prompt_logits(ids)
    print(tel.summary())

The model calls ``telemetry.layer(...)`` / ``telemetry.router(...)`` when a
Telemetry object is attached (``model.telemetry``); captured CUDA graphs never
run with it attached (the hooks read device tensors back to the host).

Counterparts of the reference's validation block: layer_rms(), router_entropy(),
expert_fire_counts() and activation absmax telemetry (engines/glm5-moe-nvfp4-2b/
src/model.h:192-258).
"""
from __future__ import annotations

import math

import torch


class Telemetry:
    def __init__(self, model):
        self.model = model
        self.rms: dict = {}
        self.absmax: dict = {}
        self.entropy: dict = {}
        self.fire: dict = {}

    def __enter__(self):
        self.model.telemetry = self
        return self

    def __exit__(self, *exc):
        self.model.telemetry = None
        return False

    # ------------------------------------------------------------------ hooks
    def layer(self, i, x: torch.Tensor):
        xf = x.float()
        self.rms[i] = float(xf.pow(2).mean().sqrt())
        self.absmax[i] = float(xf.abs().max())

    def router(self, i, logits: torch.Tensor, num_experts: int, sigmoid: bool, ids: torch.Tensor | None = None):
        lg = logits[:, :num_experts].float()
        p = torch.sigmoid(lg) if sigmoid else torch.softmax(lg, -1)
        p = p / p.sum(-1, keepdim=True).clamp_min(1e-30)
        ent = -(p * p.clamp_min(1e-30).log()).sum(-1)
        self.entropy[i] = float(ent.mean() / math.log(num_experts))  # normalised to [0, 1]
        if ids is not None:
            sel = ids[(ids >= 0) & (ids < num_experts)].long()
            c = torch.bincount(sel, minlength=num_experts).cpu()
            self.fire[i] = c if i not in self.fire else self.fire[i] + c

    # ------------------------------------------------------------------ report
    def fire_histogram(self) -> torch.Tensor:
        """Expert fire counts summed over layers [num_experts] (input of expert balancing)."""
        if not self.fire:
            return torch.zeros(0, dtype=torch.long)
        return torch.stack(list(self.fire.values())).sum(0)

    def summary(self) -> dict:
        return {"layer_rms": {str(k): round(v, 5) for k, v in self.rms.items()},
                "layer_absmax": {str(k): round(v, 4) for k, v in self.absmax.items()},
                "router_entropy": {str(k): round(v, 4) for k, v in self.entropy.items()},
                "expert_fires": int(sum(int(v.sum()) for v in self.fire.values()))}
