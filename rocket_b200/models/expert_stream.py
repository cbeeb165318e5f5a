"""Streamed routed experts: MoE layers whose routed experts live in pinned host
memory, with a bounded number of device slots per layer (LRU, native
``_rt.ExpertSlotCache``).

For a model whose experts do not fit next to the KV cache (or to trade expert
residency for KV pages), ``MoELM.enable_expert_streaming(slots)`` before the
weights are built moves every MoE layer's routed experts to host memory as the
layer is built, so device memory holds one layer's experts at most during
loading.  The shared experts stay on the device after the slots.

Per MoE layer and step: the router runs as usual; the distinct local experts it
picked are read back (one device -> host sync per layer), the slot cache splits
them into passes of at most `slots` experts, each pass's missing experts are
copied host -> device into their slots, the routing ids are rewritten to slot
ids (experts outside the pass become -1, which the plan skips), and the grouped
GEMMs + combine run once per pass (a later pass accumulates onto the first).
With enough slots for one step's experts there is a single pass and the result
equals the resident model's bit for bit; more passes add one bf16 rounding of
the residual per extra pass.

The host reads make this an eager-only mode: the engine turns CUDA graphs off.
Counterpart of the streamed half of the reference's weight store (bounded device
LRU of expert slots: engines/glm5-moe-nvfp4-2b/src/weights.h:1-16, :149-204).
"""
from __future__ import annotations

import torch


def _pinned(n: int, dtype) -> torch.Tensor:
    t = torch.empty(n, dtype=dtype)
    return t.pin_memory() if torch.cuda.is_available() else t


class _HostExperts:
    """One stacked NVFP4 weight's routed experts in pinned host memory."""

    def __init__(self, w, n_routed: int):
        E = w.num_experts
        self.n, self.k = w.n, w.k
        self.pk = w.packed.numel() // E    # bytes of one expert's packed rows
        self.sf = w.sf.numel() // E        # bytes of one expert's scale atoms
        self.gs = w.gscale.numel() // E    # fp32 row scales of one expert
        self.packed = _pinned(n_routed * self.pk, torch.uint8)
        self.sfb = _pinned(n_routed * self.sf, torch.uint8)
        self.gscale = _pinned(n_routed * self.gs, torch.float32)
        self.packed.copy_(w.packed.view(-1)[:n_routed * self.pk])
        self.sfb.copy_(w.sf.view(-1)[:n_routed * self.sf])
        self.gscale.copy_(w.gscale.view(-1)[:n_routed * self.gs])

    def load(self, dev_w, e: int, s: int):
        """Copy routed expert `e` into device slot `s` (three async copies)."""
        dev_w.packed.view(-1)[s * self.pk:(s + 1) * self.pk].copy_(self.packed[e * self.pk:(e + 1) * self.pk],
                                                                    non_blocking=True)
        dev_w.sf.view(-1)[s * self.sf:(s + 1) * self.sf].copy_(self.sfb[e * self.sf:(e + 1) * self.sf],
                                                              non_blocking=True)
        dev_w.gscale.view(-1)[s * self.gs:(s + 1) * self.gs].copy_(self.gscale[e * self.gs:(e + 1) * self.gs],
                                                                  non_blocking=True)

    def nbytes(self) -> int:
        return self.packed.numel() + self.sfb.numel() + 4 * self.gscale.numel()


class ExpertStreamer:
    def __init__(self, n_routed: int, n_shared: int, slots: int, device):
        if slots < 1:
            raise ValueError("expert streaming needs at least one slot per layer")
        self.n_routed, self.n_shared = n_routed, n_shared
        self.slots = min(slots, n_routed)
        self.dev = device
        self.layers: dict[int, tuple] = {}   # id(layer) -> (host w13, host w2, cache)
        self.bytes_loaded = 0

    def adopt(self, L):
        """Move layer L's routed experts to the host; L.w13 / L.w2 become slot weights
        (`slots` routed slots followed by the shared experts)."""
        from .. import _rt
        from ..ops import NvFp4Weight
        hosts, devs = [], []
        S, R = self.slots, self.n_routed
        for w in (L.w13, L.w2):
            h = _HostExperts(w, R)
            n_dev = S + self.n_shared
            d = NvFp4Weight(torch.empty(n_dev * w.n, w.k // 2, dtype=torch.uint8, device=self.dev),
                            torch.empty(n_dev * h.sf, dtype=torch.uint8, device=self.dev),
                            torch.empty(n_dev * h.gs, dtype=torch.float32, device=self.dev), w.n, w.k, n_dev)
            if self.n_shared:
                d.packed.view(-1)[S * h.pk:].copy_(w.packed.view(-1)[R * h.pk:])
                d.sf.view(-1)[S * h.sf:].copy_(w.sf.view(-1)[R * h.sf:])
                d.gscale.view(-1)[S * h.gs:].copy_(w.gscale.view(-1)[R * h.gs:])
            hosts.append(h)
            devs.append(d)
        L.w13, L.w2 = devs
        self.layers[id(L)] = (hosts[0], hosts[1], _rt.ExpertSlotCache(self.n_routed, self.slots))

    def host_bytes(self) -> int:
        return sum(a.nbytes() + b.nbytes() for a, b, _ in self.layers.values())

    def passes(self, L, ids: torch.Tensor):
        """Yield, per pass, the routing ids rewritten to slot ids (a device tensor like
        `ids`) after the pass's host -> device copies have been issued."""
        h13, h2, cache = self.layers[id(L)]
        R, S = self.n_routed, self.slots
        routed = ids[(ids >= 0) & (ids < R)]
        needed = torch.unique(routed).cpu().tolist()   # the one host sync of the layer
        safe = ids.clamp(min=0).long()
        for i, (remap, loads) in enumerate(cache.plan(needed)):
            for e, s in loads:
                h13.load(L.w13, e, s)
                h2.load(L.w2, e, s)
            self.bytes_loaded += len(loads) * (h13.pk + h13.sf + 4 * h13.gs + h2.pk + h2.sf + 4 * h2.gs)
            shared = list(range(S, S + self.n_shared)) if i == 0 else [-1] * self.n_shared
            table = torch.tensor(list(remap) + shared, dtype=torch.int32).to(self.dev, non_blocking=True)
            yield torch.where(ids >= 0, table[safe], torch.full_like(ids, -1))

    def stats(self) -> dict:
        out = {"slots": self.slots, "layers": len(self.layers), "host_bytes": self.host_bytes(),
               "bytes_loaded": self.bytes_loaded, "hits": 0, "misses": 0, "evictions": 0, "passes": 0}
        for _, _, c in self.layers.values():
            for k, v in c.stats().items():
                out[k] += v
        return out
