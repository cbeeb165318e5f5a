"""Debug checksum taps: per-step digests of device state for run-to-run comparison.

    ROCKET_CHECKSUM=kv,hidden,spec python -m rocket_b200 generate ...   # or
    eng.checksums = ChecksumTap(eng, {"kv", "hidden", "spec"}, "taps.jsonl")

After every engine step the tap records a 64-bit digest of the selected state:
``kv`` the KV pages of the running sequences (every attention layer; DeltaNet
recurrent state of their slots on hybrid models), ``hidden`` the last layer's hidden
rows of the step, ``spec`` the packed step outputs (sampled ids, accepted counts,
drafts).  Two runs of the same workload must produce identical streams: the first
differing step localizes a race or a nondeterministic reduction to one step and one
state family (the bisection the reference does with ROCKET_KV_CHECKSUM /
ROCKET_LHC_CHECKSUM / ROCKET_SPEC_CHECKSUM, engines/glm5-moe-nvfp4-2b/src/model.cu).

The digest is computed on the device (int64 arithmetic on the raw bits: a weighted sum
with position-dependent odd multipliers, so permutations and bit flips both change it)
and read back once per step; taps cost a few small kernels and are for debugging only.
"""
from __future__ import annotations

import json
import os

import torch

_M = (1 << 61) - 1


def digest(t: torch.Tensor) -> int:
    """64-bit digest of a device tensor's bytes (order- and value-sensitive)."""
    if t.numel() == 0:
        return 0
    b = t.contiguous().view(torch.uint8).reshape(-1)
    pad = (-b.numel()) % 4
    if pad:
        b = torch.cat([b, torch.zeros(pad, dtype=torch.uint8, device=b.device)])
    w = b.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    idx = torch.arange(w.numel(), device=w.device, dtype=torch.int64)
    mul = (idx * 2654435761 + 0x9E3779B1) | 1          # odd, position dependent
    h1 = ((w * mul) % _M).sum() % _M
    h2 = ((w ^ (idx * 40503)) % _M).sum() % _M
    return int(((h1 << 3) ^ h2).item()) & ((1 << 64) - 1)


class ChecksumTap:
    FAMILIES = ("kv", "hidden", "spec")

    def __init__(self, engine, families, path: str | None = None):
        bad = set(families) - set(self.FAMILIES)
        if bad:
            raise ValueError(f"unknown checksum families {sorted(bad)}")
        self.engine, self.families, self.path = engine, set(families), path
        self.records: list[dict] = []
        self._fh = open(path, "w") if path else None

    @staticmethod
    def from_env(engine):
        v = os.environ.get("ROCKET_CHECKSUM")
        if not v:
            return None
        return ChecksumTap(engine, [x for x in v.split(",") if x], os.environ.get("ROCKET_CHECKSUM_FILE"))

    def after_step(self, sched, T: int):
        eng, m = self.engine, self.engine.model
        rec = {"step": eng.stats.steps}
        if "kv" in self.families:
            pages = sorted({p for s in sched for p in eng.kv.pages(s.req.rid)})
            if pages:
                idx = torch.tensor(pages, dtype=torch.long, device=m.dev)
                rec["kv"] = [digest(c.index_select(1, idx)) for c in m.page_caches() if c.numel()]
            if eng.hybrid:
                slots = torch.tensor([eng.slot_of[s.req.rid] for s in sched if s.req.rid in eng.slot_of],
                                     dtype=torch.long, device=m.dev)
                if slots.numel():
                    rec["dn_state"] = digest(m.dn_buf.state.index_select(1, slots))
        if "hidden" in self.families:
            rec["hidden"] = digest(m.x[:T])
        if "spec" in self.families:
            rec["spec"] = digest(m.step_out)
        self.records.append(rec)
        if self._fh:
            self._fh.write(json.dumps(rec) + "\n")
            self._fh.flush()

    def close(self):
        if self._fh:
            self._fh.close()
            self._fh = None


def first_divergence(a: list[dict], b: list[dict]):
    """(step index, family) of the first record where two tap streams differ, or None."""
    for i, (x, y) in enumerate(zip(a, b)):
        for k in sorted(set(x) | set(y)):
            if k != "step" and x.get(k) != y.get(k):
                return i, k
    if len(a) != len(b):
        return min(len(a), len(b)), "length"
    return None
